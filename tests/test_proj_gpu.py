"""GPU parity of the fused attention projections (proj_sm100.cu) against the
CPU oracle and the reference-generated fixture, through the C ABI.

Tolerance: the projection is rounded to fp16 before any epilogue math, as the
reference's fp16 linear output; the GPU's fp32 accumulation order differs from
numpy's, so a rounding can land one fp16 ulp away (2^-11 relative), which the
norm and rotation carry through.  Outputs are compared after fp16 storage with
|gpu - oracle| <= 2e-3 + 2e-3 |oracle|; the gated residual (fp32) with
|gpu - oracle| <= 1e-5 + 2e-3 |gate * branch|.  Both also bound the MEAN error
by a quarter of an fp16 ulp of the mean magnitude (2^-13 mean |oracle|, plus
1e-6): rounding that lands one ulp away at scattered elements passes, a
systematic one-ulp bias over the output does not.
"""
import os

import numpy as np
import pytest

from oracle import attn_oracle as ora
from oracle import inputs
from tests.conftest import GOLDEN
from tests.gpu_util import assert_parity, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ex():
    from animaxs_b200 import AttentionExecutor
    e = AttentionExecutor(0)
    yield e
    e.close()


@pytest.fixture(scope="module")
def pj(ex):
    from animaxs_b200 import ProjectionExecutor
    return ProjectionExecutor(ex)


def _close_fp16(got, want, what):
    want16 = ora.to_fp16_storage(want)
    err = np.abs(np.asarray(got, dtype=np.float32) - want16)
    bound = 2e-3 + 2e-3 * np.abs(want16)
    bad = err > bound
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    assert not bad.any(), f"{what}: {bad.sum()} elements out of tolerance, worst {err.max():.3e}"
    mean_bound = 2.0 ** -13 * float(np.abs(want16).mean()) + 1e-6
    assert err.mean() <= mean_bound, f"{what}: mean-abs {err.mean():.3e} > {mean_bound:.3e}"


def _close_gate(got, want, term, what):
    err = np.abs(got - want)
    bad = err > 1e-5 + 2e-3 * np.abs(term)
    assert not bad.any(), f"{what}: {bad.sum()} elements out of tolerance, worst {err.max():.3e}"
    mean_bound = 2.0 ** -13 * float(np.abs(term).mean()) + 1e-6
    assert err.mean() <= mean_bound, f"{what}: mean-abs {err.mean():.3e} > {mean_bound:.3e}"


def test_golden_fixture(pj):
    """The reference's own linear + rms_norm + dit_rope + apply_split_half_rope
    and gated residual (tests/golden/proj_small.npz)."""
    import torch
    g = np.load(os.path.join(GOLDEN, "proj_small.npz"))
    seed, images, tokens, k, qh, kh, vc = (int(v) for v in g["qkv_meta"])
    x, w, qw, kw = inputs.proj_qkv(seed, images=images, tokens=tokens, k=k, q_heads=qh, k_heads=kh, v_cols=vc)
    rope = to_dev(ora.dit_rope_table(1, 8, 8))
    for mode, key in (("rms_rope", "qkv_rope_out"), ("rms", "qkv_rms_out")):
        out = pj.qkv(to_dev(x), to_dev(w), q_cols=qh * 128, k_cols=kh * 128, qk_norm=mode,
                     q_norm_weight=to_dev(qw), k_norm_weight=to_dev(kw), rope_table=rope, tokens=tokens)
        torch.cuda.synchronize()
        _close_fp16(out.float().cpu().numpy(), g[key], f"golden qkv {mode}")
    seed, images, tokens, k, n = (int(v) for v in g["gate_meta"])
    xg, wg, res, gate = inputs.proj_gate(seed, images=images, tokens=tokens, k=k, n=n)
    r = to_dev(res)
    pj.out_gate_add(to_dev(xg), to_dev(wg), r, to_dev(gate), tokens=tokens)
    torch.cuda.synchronize()
    _close_gate(r.cpu().numpy(), g["gate_out"], g["gate_out"] - res, "golden gate add")


@pytest.mark.parametrize("images,tokens,k,qh,kh,vc", [
    (1, 1, 64, 1, 1, 128),        # one row
    (1, 129, 200, 1, 1, 128),     # ragged rows, k not a multiple of 64 (TMA zero fill)
    (2, 300, 256, 2, 2, 384),     # n = 1024 (a 256-wide tile split over q / k heads)
    (3, 256, 512, 3, 1, 128),     # n = 640: last tile half out of range
    (1, 4096, 2048, 16, 16, 2048),  # DiT self-attention q|k|v: 4096 x 6144 x 2048
])
def test_qkv_norm_rope(pj, images, tokens, k, qh, kh, vc):
    import torch
    x, w, qw, kw = inputs.proj_qkv(images * tokens + k + qh, images=images, tokens=tokens, k=k, q_heads=qh,
                                   k_heads=kh, v_cols=vc)
    grid = {1: (1, 1, 1), 129: (1, 3, 43), 300: (1, 15, 20), 256: (1, 16, 16), 4096: (1, 64, 64)}[tokens]
    table = ora.dit_rope_table(*grid)
    out = pj.qkv(to_dev(x), to_dev(w), q_cols=qh * 128, k_cols=kh * 128, qk_norm="rms_rope",
                 q_norm_weight=to_dev(qw), k_norm_weight=to_dev(kw), rope_table=to_dev(table), tokens=tokens)
    torch.cuda.synchronize()
    want = ora.qkv_norm_projection(x, w, q_cols=qh * 128, k_cols=kh * 128, q_norm_weight=qw,
                                   k_norm_weight=kw, rope_table=table, tokens=tokens)
    _close_fp16(out.float().cpu().numpy(), want, f"qkv {images}x{tokens} k={k}")


def test_cross_q_rms_and_plain_linear(pj):
    """Cross-attention q (RMSNorm only, no k heads) and the plain projection."""
    import torch
    x, w, qw, _ = inputs.proj_qkv(5, images=1, tokens=777, k=1024, q_heads=16, k_heads=0, v_cols=0)
    out = pj.qkv(to_dev(x), to_dev(w), q_cols=2048, k_cols=0, qk_norm="rms", q_norm_weight=to_dev(qw))
    lin = pj.linear(to_dev(x), to_dev(w))
    torch.cuda.synchronize()
    _close_fp16(out.float().cpu().numpy(),
                ora.qkv_norm_projection(x, w, q_cols=2048, k_cols=0, qk_norm="rms", q_norm_weight=qw),
                "cross q rms")
    _close_fp16(lin.float().cpu().numpy(), ora.linear_fp16(x, w), "plain linear")


def test_strided_rows(pj):
    """x and out as row-strided views (a [m, 3n] buffer's middle block)."""
    import torch
    x, w, _, _ = inputs.proj_qkv(9, images=1, tokens=200, k=256, q_heads=0, k_heads=0, v_cols=512)
    xb = torch.zeros(200, 384, dtype=torch.float16, device="cuda")
    xb[:, 64:320] = to_dev(x)
    ob = torch.full((200, 3 * 512), 7.0, dtype=torch.float16, device="cuda")
    pj.linear(xb[:, 64:320], to_dev(w), ob[:, 512:1024])
    torch.cuda.synchronize()
    _close_fp16(ob[:, 512:1024].float().cpu().numpy(), ora.linear_fp16(x, w), "strided")
    assert torch.all(ob[:, :512] == 7.0) and torch.all(ob[:, 1024:] == 7.0)


@pytest.mark.parametrize("images,tokens,k,n", [(1, 1, 64, 256), (2, 333, 256, 512), (2, 4096, 2048, 2048)])
def test_out_gate_add(pj, images, tokens, k, n):
    """residual += fp16(x w^T) * gate[image], twice (accumulates in place)."""
    import torch
    x, w, res, gate = inputs.proj_gate(images * 7 + tokens, images=images, tokens=tokens, k=k, n=n)
    r = to_dev(res)
    xd, wd, gd = to_dev(x), to_dev(w), to_dev(gate)
    pj.out_gate_add(xd, wd, r, gd, tokens=tokens)
    pj.out_gate_add(xd, wd, r, gd, tokens=tokens)
    torch.cuda.synchronize()
    once = ora.gate_add_projection(res, x, w, gate, tokens=tokens)
    twice = ora.gate_add_projection(once, x, w, gate, tokens=tokens)
    _close_gate(r.cpu().numpy(), twice, 2 * (once - res), f"gate add {images}x{tokens} n={n}")


def test_fused_projection_feeds_attention(ex, pj):
    """q|k|v from the fused QKV_NORM projection into attention (qk_norm none)
    agrees with the unfused chain: plain projection, then attention's own fused
    rms + rope3d prologue."""
    import torch
    x, w, qw, kw = inputs.proj_qkv(31, images=1, tokens=1024, k=2048, q_heads=16, k_heads=16, v_cols=2048)
    rope = to_dev(ora.dit_rope_table(1, 32, 32))
    xd, wd, qwd, kwd = to_dev(x), to_dev(w), to_dev(qw), to_dev(kw)
    fused = pj.qkv(xd, wd, q_cols=2048, k_cols=2048, q_norm_weight=qwd, k_norm_weight=kwd, rope_table=rope)
    plain = pj.linear(xd, wd)
    view = lambda t, c0: t[:, c0:c0 + 2048].view(1, 1024, 16, 128)  # noqa: E731
    o1 = ex.attention(view(fused, 0), view(fused, 2048), view(fused, 4096))
    o2 = ex.attention(view(plain, 0), view(plain, 2048), view(plain, 4096), qk_norm="rms_rope",
                      rope_table=rope, q_norm_weight=qwd, k_norm_weight=kwd)
    torch.cuda.synchronize()
    a, b = o1.float().cpu().numpy(), o2.float().cpu().numpy()
    assert np.abs(a - b).max() <= 2e-3, np.abs(a - b).max()
    q = ora.qkv_norm_projection(x, w, q_cols=2048, k_cols=2048, q_norm_weight=qw, k_norm_weight=kw,
                                rope_table=ora.dit_rope_table(1, 32, 32))
    qkv = ora.to_fp16_storage(q).reshape(1, 1024, 3, 16, 128)
    assert_parity(a, ora.attention(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]), what="fused projection -> attention")
