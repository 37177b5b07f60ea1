"""GPU parity of the W8 / W4 weight decode (dequant_sm100.cu) and of the
projections that take quantized weights, through the C ABI.

The decode is integer-in, fp16-out arithmetic with a fixed rounding sequence,
so it is compared BIT-EXACT: against the reference's own decoders on weights
packed by the reference's own quantizer (tests/golden/quant_small.npz) and
against the oracle's restatement on seeded codes.  A projection with
quantized weights must equal, bit for bit, the same projection given the
decoded fp16 weight (the GEMM is the same kernel on the same operand); against
the oracle it is held to the fp16 projection tolerance
|gpu - oracle| <= 2e-3 + 2e-3 |oracle|.
"""
import os

import numpy as np
import pytest

from oracle import attn_oracle as ora
from oracle import inputs
from tests.conftest import GOLDEN
from tests.gpu_util import to_dev

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


def _qw(packed, scale, zero, bits, k):
    import torch
    from animaxs_b200 import QuantizedWeight
    return QuantizedWeight(torch.from_numpy(np.ascontiguousarray(packed)).cuda(),
                           torch.from_numpy(np.ascontiguousarray(scale)).cuda(),
                           torch.from_numpy(np.ascontiguousarray(zero)).cuda(), bits, k)


def _bits_equal(got, want, what):
    got = np.asarray(got, dtype=np.float16)
    want = np.asarray(want, dtype=np.float16)
    assert got.shape == want.shape, what
    diff = got.view(np.uint16) != want.view(np.uint16)
    assert not diff.any(), f"{what}: {diff.sum()} values differ, first at {np.argwhere(diff)[0]}"


def _close_fp16(got, want, what):
    want16 = ora.to_fp16_storage(want)
    err = np.abs(np.asarray(got, dtype=np.float32) - want16)
    bad = err > 2e-3 + 2e-3 * np.abs(want16)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    assert not bad.any(), f"{what}: {bad.sum()} elements out of tolerance, worst {err.max():.3e}"
    # mean error under a quarter fp16 ulp of the mean magnitude: no systematic bias
    mean_bound = 2.0 ** -13 * float(np.abs(want16).mean()) + 1e-6
    assert err.mean() <= mean_bound, f"{what}: mean-abs {err.mean():.3e} > {mean_bound:.3e}"


def test_golden_decode(pj):
    """Codes from the reference's quantizer (plain, W4 range search, ragged last
    group, odd W4 rows of 65 bytes) decode to the reference decoders' fp16."""
    import torch
    g = np.load(os.path.join(GOLDEN, "quant_small.npz"))
    for name in ("w8", "w4", "w4opt", "w4wide"):
        bits, rows, k, _opt, _seed = (int(v) for v in g[name + "_meta"])
        out = pj.dequant(_qw(g[name + "_packed"], g[name + "_scale"], g[name + "_zero"], bits, k))
        torch.cuda.synchronize()
        _bits_equal(out.cpu().numpy(), g[name + "_decoded_half"], f"golden {name}")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("rows,k,pad", [
    (1, 1, 0),          # a single value
    (3, 7, 0),          # one partial chunk per row
    (5, 63, 1),         # ragged group, odd W4 row bytes, padded rows
    (7, 65, 3),         # a second group of one column
    (64, 1024, 0),      # aligned rows: the vector path only
    (33, 1000, 5),      # unaligned packed rows: byte path for most rows
    (6144, 2048, 0),    # the DiT self-attention q|k|v weight
])
def test_decode_matches_oracle(pj, bits, rows, k, pad):
    import torch
    need = (k + 1) // 2 if bits == 4 else k
    packed, scale, zero = inputs.quant_weight(100 + rows + k, rows, k, bits, packed_stride=need + pad)
    out = pj.dequant(_qw(packed, scale, zero, bits, k))
    torch.cuda.synchronize()
    _bits_equal(out.cpu().numpy(), ora.dequant_to_half(packed, scale, zero, bits=bits, k=k),
                f"W{bits} {rows}x{k} pad {pad}")


def test_decode_into_strided_unaligned_output(pj):
    """A destination with a row stride that is not a multiple of 8 halves and a
    start 2 bytes off 16: the scalar store path; the gaps stay untouched."""
    import torch
    rows, k = 9, 200
    packed, scale, zero = inputs.quant_weight(5, rows, k, 4)
    buf = torch.full((rows * 203 + 1,), 7.0, dtype=torch.float16, device="cuda")
    out = buf[1:].view(rows, 203)[:, :k]
    pj.dequant(_qw(packed, scale, zero, 4, k), out=out)
    torch.cuda.synchronize()
    full = buf[1:].view(rows, 203).cpu().numpy()
    _bits_equal(full[:, :k], ora.dequant_to_half(packed, scale, zero, bits=4, k=k), "strided W4")
    assert (full[:, k:] == 7.0).all() and buf[0].item() == 7.0


def test_decode_extreme_codes(pj):
    """Codes 0 and qmax with fp16 scales/zeros at the edges of their range
    (subnormal scale, large zero, negative scale): still bit-exact."""
    import torch
    rows, k = 4, 128
    for bits, qmax in ((8, 255), (4, 15)):
        q = np.zeros((rows, k), dtype=np.uint8)
        q[:, 1::2] = qmax
        packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8) if bits == 4 else q
        scale = np.array([[6e-8, 1e-4], [0.5, 60.0], [-0.01, 1.0], [1.0, 2.0]], dtype=np.float16)
        zero = np.array([[0.0, -1e-3], [-30000.0, 100.0], [0.25, -0.25], [65000.0, -65000.0]], dtype=np.float16)
        out = pj.dequant(_qw(packed, scale, zero, bits, k))
        torch.cuda.synchronize()
        _bits_equal(out.cpu().numpy(), ora.dequant_to_half(packed, scale, zero, bits=bits, k=k), f"extreme W{bits}")


def test_golden_quantized_projection(pj):
    """x times the reference-quantized W4 weight, against the reference's
    linear on its decoded weight (tests/golden/quant_small.npz)."""
    import torch
    g = np.load(os.path.join(GOLDEN, "quant_small.npz"))
    seed, m, k = (int(v) for v in g["proj_w4_meta"])
    x = to_dev(inputs.proj_x(seed, m, k))
    w = _qw(g["w4wide_packed"], g["w4wide_scale"], g["w4wide_zero"], 4, k)
    out = pj.linear(x, w)
    torch.cuda.synchronize()
    _close_fp16(out.float().cpu().numpy(), g["proj_w4_out"], "golden W4 projection")


@pytest.mark.parametrize("bits", [4, 8])
def test_quantized_equals_fp16_on_decoded_weight(pj, bits):
    """DiT q|k|v at full size (4096 x 6144 x 2048, RMSNorm + RoPE epilogue):
    the quantized call is bit-identical to the fp16 call on the decoded
    weight, and the decoded weight is bit-exact to the oracle."""
    import torch
    k, n, tokens = 2048, 6144, 4096
    packed, scale, zero = inputs.quant_weight(40 + bits, n, k, bits)
    w = _qw(packed, scale, zero, bits, k)
    x = to_dev(inputs.proj_x(41, tokens, k))
    rope = to_dev(ora.dit_rope_table(1, 64, 64))
    qn = to_dev(np.linspace(0.5, 1.5, 128, dtype=np.float32).astype(np.float16))
    kn = to_dev(np.linspace(1.5, 0.5, 128, dtype=np.float32).astype(np.float16))
    kw = dict(q_cols=2048, k_cols=2048, q_norm_weight=qn, k_norm_weight=kn, rope_table=rope, tokens=tokens)
    got = pj.qkv(x, w, **kw)
    wdec = pj.dequant(w)
    ref = pj.qkv(x, wdec, **kw)
    torch.cuda.synchronize()
    _bits_equal(wdec.cpu().numpy(), ora.dequant_to_half(packed, scale, zero, bits=bits, k=k), "decoded weight")
    assert torch.equal(got, ref), "quantized projection differs from the fp16 projection on the decoded weight"


@pytest.mark.parametrize("bits", [4, 8])
def test_quantized_qkv_and_gate_add_match_oracle(pj, bits):
    import torch
    images, tokens, k = 2, 64, 256
    m = images * tokens
    x = inputs.proj_x(50 + bits, m, k)
    packed, scale, zero = inputs.quant_weight(60 + bits, 768, k, bits)
    wdec = ora.dequant_to_half(packed, scale, zero, bits=bits, k=k)
    qw = np.linspace(0.8, 1.2, 128, dtype=np.float32).astype(np.float16)
    tab = ora.dit_rope_table(1, 8, 8)
    out = pj.qkv(to_dev(x), _qw(packed, scale, zero, bits, k), q_cols=256, k_cols=256, qk_norm="rms_rope",
                 q_norm_weight=to_dev(qw), k_norm_weight=to_dev(qw), rope_table=to_dev(tab), tokens=tokens)
    torch.cuda.synchronize()
    want = ora.qkv_norm_projection(x, wdec, q_cols=256, k_cols=256, q_norm_weight=qw, k_norm_weight=qw,
                                   rope_table=tab, tokens=tokens)
    _close_fp16(out.float().cpu().numpy(), want, f"W{bits} q|k|v")
    # out-projection + gated residual with an odd-stride W4/W8 weight
    need = (k + 1) // 2 if bits == 4 else k
    packed, scale, zero = inputs.quant_weight(70 + bits, 256, k, bits, packed_stride=need + 3)
    wdec = ora.dequant_to_half(packed, scale, zero, bits=bits, k=k)
    res = np.random.default_rng(bits).standard_normal((m, 256)).astype(np.float32)
    gate = np.random.default_rng(bits + 1).standard_normal((images, 256)).astype(np.float32)
    r = to_dev(res)
    pj.out_gate_add(to_dev(x), _qw(packed, scale, zero, bits, k), r, to_dev(gate), tokens=tokens)
    torch.cuda.synchronize()
    want = ora.gate_add_projection(res, x, wdec, gate, tokens=tokens)
    term = want - res
    err = np.abs(r.cpu().numpy() - want)
    assert not (err > 1e-5 + 2e-3 * np.abs(term)).any(), f"W{bits} gate add: worst {err.max():.3e}"
