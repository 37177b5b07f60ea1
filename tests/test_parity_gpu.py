"""GPU parity: the tcgen05 attention path against the CPU oracle and the
reference-generated golden fixtures, through the C ABI (ctypes)."""
import os

import numpy as np
import pytest

from oracle import attn_oracle as ora
from oracle import inputs
from tests.conftest import GOLDEN
from tests.gpu_util import assert_parity, run_case, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ex():
    from animaxs_b200 import AttentionExecutor
    e = AttentionExecutor(0)
    yield e
    e.close()


def _golden(name):
    return np.load(os.path.join(GOLDEN, name))


# ------------------------------------------------------------------ configs --
def test_config1_dit_self_1024(ex):
    case = inputs.dit_self(seed=0, grid=(1, 32, 32))
    out = run_case(ex, case)
    assert_parity(out, case.oracle(), what="config 1")
    g = _golden("attn_configs.npz")
    rows = g["cfg1_rows"]
    assert_parity(out[:, rows], g["cfg1_out"], what="config 1 vs reference golden")


@pytest.mark.parametrize("masked", [True, False])
def test_config2_dit_cross(ex, masked):
    case = inputs.dit_cross(seed=0, kv_valid=128 if masked else None)
    out = run_case(ex, case)
    assert_parity(out, case.oracle(), what=f"config 2 masked={masked}")
    g = _golden("attn_configs.npz")
    key = "cfg2_masked" if masked else "cfg2_unmasked"
    assert_parity(out[:, g[key + "_rows"]], g[key + "_out"], what="config 2 vs golden")


@pytest.mark.parametrize("layer", list(range(28)))
def test_config3_qwen_prefill(ex, layer):
    case = inputs.qwen_prefill(layer=layer)
    out = run_case(ex, case, layout="head")
    assert_parity(out, case.oracle(), what=f"config 3 layer {layer}")
    if layer in (0, 27):
        g = _golden("attn_configs.npz")
        key = f"cfg3_l{layer}"
        assert_parity(out[:, g[key + "_rows"]], g[key + "_out"], what="config 3 vs golden")


def test_config4_subset(ex):
    g = _golden("attn_configs.npz")
    for prompt in (0, 7):
        for step in (0, 7):
            for block in (0, 27):
                sc, cc = inputs.workload_block(prompt, step, block)
                tag = f"cfg4_p{prompt}_s{step}_b{block}"
                for case, kind in ((sc, "self"), (cc, "cross")):
                    rows = g[f"{tag}_{kind}_rows"]
                    out = run_case(ex, case, rows=rows)
                    assert_parity(out, g[f"{tag}_{kind}_out"], what=f"{tag} {kind}")


def test_config5_dit_self_16k(ex):
    case = inputs.dit_self(seed=0, grid=(1, 128, 128))
    g = _golden("attn_configs.npz")
    rows = g["cfg5_rows"]
    out = run_case(ex, case, rows=rows)
    assert_parity(out, g["cfg5_out"], what="config 5 vs golden")
    extra = np.array([7, 4097, 9999, 15000])
    full = run_case(ex, case)
    assert_parity(full[:, extra], case.oracle(rows=extra), what="config 5 extra rows")


# ------------------------------------------------------ small golden cases --
SMALL = {
    "dit_self_256": lambda: inputs.dit_self(seed=10, grid=(1, 16, 16), heads=2),
    "dit_cross_192x96_valid40": lambda: inputs.dit_cross(seed=11, q_len=192, kv_len=96, heads=2, kv_valid=40),
    "dit_cross_130x200": lambda: inputs.dit_cross(seed=12, q_len=130, kv_len=200, heads=2, kv_valid=None),
    "qwen_160_h4kv2_valid100": lambda: inputs.qwen_prefill(layer=0, seq_len=160, heads=4, kv_heads=2, valid=100),
}


@pytest.mark.parametrize("name", sorted(SMALL))
@pytest.mark.parametrize("layout", ["token", "head"])
def test_small_golden(ex, name, layout):
    case = SMALL[name]()
    out = run_case(ex, case, layout=layout)
    g = _golden("attn_small.npz")
    assert_parity(out, g[name + "_out"], what=name)


# ------------------------------------------------------------- edge cases --
@pytest.mark.parametrize("s", [1, 2, 127, 128, 129, 300, 511, 640])
@pytest.mark.parametrize("causal", [False, True])
def test_ragged_lengths(ex, s, causal):
    q, k, v = inputs.draw_qkv(100 + s, (1, s, 2, 128), (1, s, 2, 128))
    case = inputs.Case(f"ragged{s}", q, k, v, qk_norm="rms_rope",
                       rope_table=ora.rope1d_table(s, 1.0e6), causal=causal)
    out = run_case(ex, case)
    assert_parity(out, case.oracle(), what=f"S={s} causal={causal}")


@pytest.mark.parametrize("sq,sk,valid", [(1, 1, 1), (5, 700, 1), (300, 129, 129), (256, 1000, 999),
                                         (128, 4096, 4000), (77, 333, 200)])
def test_cross_shapes_and_padding(ex, sq, sk, valid):
    q, k, v = inputs.draw_qkv(sq * 7 + sk, (1, sq, 3, 128), (1, sk, 3, 128))
    case = inputs.Case("cross", q, k, v, qk_norm="rms", kv_valid_len=[valid])
    out = run_case(ex, case)
    assert_parity(out, case.oracle(), what=f"{sq}x{sk} valid {valid}")


def test_batched_per_batch_valid_lengths(ex):
    import torch
    q, k, v = inputs.draw_qkv(5, (3, 200, 2, 128), (3, 300, 2, 128))
    lens = [300, 17, 256]
    case = inputs.Case("batched", q, k, v, qk_norm="rms", kv_valid_len=lens)
    dl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = ex.attention(to_dev(q), to_dev(k), to_dev(v), qk_norm="rms", kv_valid_lens=dl)
    torch.cuda.synchronize()
    assert_parity(out.float().cpu().numpy(), case.oracle(), what="per-batch valid lengths")


def test_gqa_group_of_four_no_norm(ex):
    q, k, v = inputs.draw_qkv(9, (1, 257, 8, 128), (1, 257, 2, 128))
    case = inputs.Case("gqa4", q, k, v, causal=True)
    out = run_case(ex, case)
    assert_parity(out, case.oracle(), what="GQA 8q/2kv")


def test_output_sentinels_untouched(ex):
    """Sentinel-guarded output (pattern of MetalExecutionTests.swift:502-514)."""
    import torch
    case = inputs.dit_cross(seed=3, q_len=130, kv_len=70, heads=2, kv_valid=None)
    q, k, v = to_dev(case.q), to_dev(case.k), to_dev(case.v)
    big = torch.full((1, 130 + 2, 2, 128), 7.0, dtype=torch.float16, device="cuda")
    out = big[:, 1:131]
    ex.attention(q, k, v, out=out, qk_norm="rms")
    torch.cuda.synchronize()
    assert torch.all(big[:, 0] == 7.0) and torch.all(big[:, -1] == 7.0)
    assert_parity(out.float().cpu().numpy(), case.oracle(), what="sentinel case")


# ---------------------------------------------- reference test ports (Swift) --
def test_gqa_uses_contiguous_kv_heads(ex):
    """AttentionExecutorTests.swift:90-111 (dim 128 instead of 4)."""
    import torch
    from animaxs_b200 import DeviceBuffer  # noqa: F401
    heads, kv, d = 4, 2, 128
    q = torch.zeros(heads, 1, d, dtype=torch.float16, device="cuda")
    k = torch.zeros(kv, 1, d, dtype=torch.float16, device="cuda")
    v = torch.cat([torch.full((1, 1, d), 2.0), torch.full((1, 1, d), 9.0)]).half().cuda()
    o = torch.empty(heads, 1, d, dtype=torch.float16, device="cuda")
    ex.execute(q, k, v, o, heads=heads, query_count=1, key_count=1, head_dim=d, key_value_heads=kv)
    got = o.float().cpu().numpy().reshape(heads, d)
    assert np.all(got[:2] == 2.0) and np.all(got[2:] == 9.0)


def test_cross_attention_retains_all_512_rows_and_tail_tile(ex):
    """AttentionExecutorTests.swift:64-88: uniform scores -> (column+1)/512."""
    import torch
    qn, kn, d = 129, 512, 128
    q = torch.zeros(1, qn, d, dtype=torch.float16, device="cuda")
    k = torch.zeros(1, kn, d, dtype=torch.float16, device="cuda")
    v = torch.zeros(1, kn, d, dtype=torch.float16, device="cuda")
    v[0, kn - 1] = torch.arange(1, d + 1, dtype=torch.float16)
    o = torch.empty(1, qn, d, dtype=torch.float16, device="cuda")
    ex.execute(q, k, v, o, heads=1, query_count=qn, key_count=kn, head_dim=d)
    got = o.float().cpu().numpy()[0]
    expect = (np.arange(1, d + 1) / 512.0)
    for row in (0, 127, 128):
        np.testing.assert_allclose(got[row], expect, atol=1e-4)


def test_token_major_no_head_mixing(ex):
    """AttentionExecutorTests.swift:460-504 with headDim 128: Q=K=0 -> mean of V per head."""
    import torch
    from animaxs_b200 import AttentionInputLayout
    heads, d, rows = 2, 128, 3
    md = heads * d
    vals = np.zeros((rows, md), np.float32)
    for t in range(rows):
        for h in range(heads):
            vals[t, h * d:(h + 1) * d] = t * 10 + h + np.arange(d) / 1000.0
    zeros = torch.zeros(rows, md, dtype=torch.float16, device="cuda")
    vbuf = torch.from_numpy(vals).half().cuda()
    o = torch.empty(rows, md, dtype=torch.float16, device="cuda")
    ex.execute(zeros, zeros, vbuf, o, heads=heads, query_count=rows, key_count=rows, head_dim=d,
               layout=AttentionInputLayout.token_major(md))
    got = o.float().cpu().numpy()
    expect = vbuf.float().cpu().numpy().mean(axis=0)
    for t in range(rows):
        np.testing.assert_allclose(got[t], expect, atol=0.05)


def test_query_tile_counter(ex):
    """AttentionExecutorTests.swift:207-227: 2 heads x ceil(130/128) = 4 tiles."""
    import torch
    heads, qn, kn, d = 2, 130, 64, 128
    before = ex.attention_query_tiles
    q = torch.zeros(heads, qn, d, dtype=torch.float16, device="cuda")
    k = torch.zeros(1, kn, d, dtype=torch.float16, device="cuda")
    v = torch.ones(1, kn, d, dtype=torch.float16, device="cuda")
    o = torch.empty(heads, qn, d, dtype=torch.float16, device="cuda")
    ex.execute(q, k, v, o, heads=heads, query_count=qn, key_count=kn, head_dim=d, key_value_heads=1)
    assert ex.attention_query_tiles - before == 4
    assert np.allclose(o.float().cpu().numpy(), 1.0)


def test_full_dit_shapes_finite(ex):
    """AttentionExecutorTests.swift:427-455: self 1024/1024 and cross 1024/512, stride 2048."""
    import torch
    from animaxs_b200 import AttentionInputLayout
    md = 2048
    def vals(rows):
        idx = np.arange(rows * md)
        return torch.from_numpy(((idx * 7 + 3) % 1009 / 2000 - 0.25).astype(np.float16).reshape(rows, md)).cuda()
    q = vals(1024)
    for kn in (1024, 512):
        kv = vals(kn)
        o = torch.empty(1024, md, dtype=torch.float16, device="cuda")
        ex.execute(q, kv, kv, o, heads=16, query_count=1024, key_count=kn, head_dim=128,
                   layout=AttentionInputLayout.token_major(md))
        got = o.float()
        assert torch.isfinite(got).all() and got.abs().sum() > 0


def test_rms_rope_split_half_kernel(ex):
    """Standalone rms_rope_split_half (AnimaKernels.metal:696-729) vs the oracle."""
    import torch
    case = inputs.dit_self(seed=4, grid=(1, 16, 16), heads=3)
    x = to_dev(case.q[0])  # [S, H, 128]
    w = torch.linspace(0.5, 1.5, 128).half().cuda()
    rope = to_dev(case.rope_table)
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    ex.rms_rope_split_half(stream, x, out, w, rope, tokens=256, heads=3)
    torch.cuda.synchronize()
    ref = ora.apply_split_half_rope(ora.rms_norm_heads(case.q.astype(np.float32), w.float().cpu().numpy()),
                                    case.rope_table)[0]
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, ora.to_fp16_storage(ref), atol=4e-3, rtol=2e-3)
    out2 = torch.empty_like(x)
    ex.rmsnorm_heads_half(stream, x, out2, None, tokens=256, heads=3)
    torch.cuda.synchronize()
    ref2 = ora.rms_norm_heads(case.q.astype(np.float32))[0]
    np.testing.assert_allclose(out2.float().cpu().numpy(), ora.to_fp16_storage(ref2), atol=4e-3, rtol=2e-3)


def test_cached_cross_k_matches_fused(ex):
    """The cross-K/V cache flow (DiTBlockExecutor.swift:1105-1161): K normalised
    once (rmsnorm_heads_half) and reused, q normalised per call
    (qk_norm_targets="q"), must equal the fused q-and-k call bit for bit."""
    import torch
    case = inputs.dit_cross(seed=21, q_len=640, kv_len=512, heads=4, kv_valid=None)
    q, k, v = to_dev(case.q), to_dev(case.k), to_dev(case.v)
    wq = torch.linspace(0.8, 1.2, 128).half().cuda()
    wk = torch.linspace(1.2, 0.8, 128).half().cuda()
    fused = ex.attention(q, k, v, qk_norm="rms", q_norm_weight=wq, k_norm_weight=wk)
    k_cached = torch.empty_like(k)
    ex.rmsnorm_heads_half(torch.cuda.current_stream(), k[0], k_cached[0], wk, tokens=512, heads=4)
    cached = ex.attention(q, k_cached, v, qk_norm="rms", q_norm_weight=wq, qk_norm_targets="q")
    torch.cuda.synchronize()
    assert torch.equal(fused, cached)
    # and k-only: q pre-normalised by the caller
    q_norm = torch.empty_like(q)
    ex.rmsnorm_heads_half(torch.cuda.current_stream(), q[0], q_norm[0], wq, tokens=640, heads=4)
    konly = ex.attention(q_norm, k, v, qk_norm="rms", k_norm_weight=wk, qk_norm_targets="k")
    torch.cuda.synchronize()
    assert torch.equal(fused, konly)
    assert_parity(fused.float().cpu().numpy(),
                  ora.forward(case.q, case.k, case.v, qk_norm="rms",
                              q_norm_weight=wq.float().cpu().numpy(),
                              k_norm_weight=wk.float().cpu().numpy()),
                  what="cross with norm weights")


# ------------------------------------------- head_dim 64 (the LLM adapter) --
@pytest.mark.parametrize("target,context", [(512, None), (300, None), (512, 512), (300, 77), (1, 512)])
@pytest.mark.parametrize("layout", ["token", "head"])
def test_adapter_attention_d64(ex, target, context, layout):
    """LLMAdapterMetal.swift:361-404: 16 heads of 64, rms_rope_adapter64 on q
    and k (fused here), non-causal self- or cross-attention."""
    case = inputs.adapter_attention(seed=target + (context or 0), target_tokens=target,
                                    context_tokens=context)
    out = run_case(ex, case, layout=layout)
    assert_parity(out, case.oracle(), what=f"adapter {target}x{context} {layout}")


@pytest.mark.parametrize("s,causal", [(1, False), (129, True), (300, False), (640, True)])
def test_d64_ragged_and_causal(ex, s, causal):
    q, k, v = inputs.draw_qkv(300 + s, (2, s, 3, 64), (2, s, 3, 64))
    case = inputs.Case(f"d64_{s}", q, k, v, qk_norm="rms_rope",
                       rope_table=ora.adapter_rope_table(s), causal=causal)
    out = run_case(ex, case)
    assert_parity(out, case.oracle(), what=f"d64 S={s} causal={causal}")


def test_d64_gqa_and_padding(ex):
    q, k, v = inputs.draw_qkv(77, (1, 257, 8, 64), (1, 400, 2, 64))
    case = inputs.Case("d64_gqa_pad", q, k, v, qk_norm="rms", kv_valid_len=[333])
    out = run_case(ex, case)
    assert_parity(out, case.oracle(), what="d64 GQA 8q/2kv, valid 333 of 400")
    case = inputs.Case("d64_gqa", q, k, v)
    out = run_case(ex, case, layout="head")
    assert_parity(out, case.oracle(), what="d64 GQA, no norm, head-major")


def test_rms_rope_adapter64_kernel(ex):
    """rms_rope_adapter64 (AnimaKernels.metal:733-763) through the standalone
    rms_rope_split_half entry at head_dim 64, with a non-trivial weight."""
    import torch
    case = inputs.adapter_attention(seed=5, target_tokens=200, heads=16)
    x = to_dev(case.q[0])  # [S, H, 64]
    w = torch.linspace(0.5, 1.5, 64).half().cuda()
    rope = to_dev(case.rope_table)
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    ex.rms_rope_split_half(stream, x, out, w, rope, tokens=200, heads=16, head_dim=64)
    torch.cuda.synchronize()
    ref = ora.apply_split_half_rope(ora.rms_norm_heads(case.q.astype(np.float32), w.float().cpu().numpy()),
                                    case.rope_table)[0]
    np.testing.assert_allclose(out.float().cpu().numpy(), ora.to_fp16_storage(ref), atol=4e-3, rtol=2e-3)


def test_rejects_unsupported(ex):
    """AttentionExecutorTests.swift:404-423 and :536-562."""
    import torch
    from animaxs_b200 import AttentionInputLayout, AttentionValidationError
    buf = torch.zeros(4, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(AttentionValidationError):
        ex.execute(buf, buf, buf, buf, heads=4, query_count=4, key_count=4, head_dim=32,
                   layout=AttentionInputLayout.token_major(128))
    with pytest.raises(AttentionValidationError, match="keyValueHeads == heads"):
        ex.execute(buf, buf, buf, buf, heads=2, query_count=4, key_count=4, head_dim=64,
                   key_value_heads=1, layout=AttentionInputLayout.token_major(128))
    with pytest.raises(AttentionValidationError, match="out of bounds"):
        ex.execute(buf, buf, buf, buf, heads=1, query_count=8, key_count=4, head_dim=128)


# ------------------------------------------------------- failure detection --
def test_bounded_wait_reports_timeout_and_context_survives(ex):
    """A device-side wait that runs out (the self-test kernel waits on a
    barrier phase nothing completes, limit 50 ms) sets the status word:
    synchronize reports ANIMAXS_ERR_TIMEOUT, clears it, and the same context
    then runs attention correctly."""
    import torch
    from animaxs_b200 import AttentionTimeoutError
    stream = torch.cuda.current_stream()
    rc = ex._lib.animaxs_attn_selftest_wait_timeout(ex.handle, 50_000_000, stream.cuda_stream)
    assert rc == 0
    with pytest.raises(AttentionTimeoutError, match="bounded device-side wait"):
        ex.synchronize(stream)
    ex.synchronize(stream)  # status cleared
    case = inputs.dit_cross(seed=3, q_len=300, kv_len=200, heads=2, kv_valid=None)
    assert_parity(run_case(ex, case), case.oracle(), what="after a reported timeout")
