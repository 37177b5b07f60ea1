"""GPU: the two attention numerics of the reference's AttentionExecutor
(``numerics:``, AttentionExecutor.swift:97-110).

``fp32ScoresAndSoftmax`` is the reference's diagnostic mode (encodeFP32,
:325-405): fp32 scores, fp32 softmax, fp32 probabilities times fp16 V
(AnimaKernels.metal:1105-1185); the reference measured it against an
independent reference at max-abs 2.40e-4 where legacy reached 1.19e-3
(TEST_MATRIX.md, "Attention numerics").  Here the fp32 probabilities enter
the tensor-core product as P_hi + P_lo (two fp16 terms), so before the final
fp16 store the result is accurate to ~1e-6 relative, and the stored output
must be the fp32 oracle rounded to fp16, give or take rounding at a tie:

    |gpu - oracle| <= 0.5 * ulp_fp16(the larger of the two) + 4e-6 * (1 + |oracle|)

The oracle here runs on the q and k that the library's own RMSNorm (+ RoPE)
kernels produced (fp16, as the reference's rms_rope_split_half writes them),
so that the bound measures the attention arithmetic alone.

Legacy numerics (fp16 P) stay at the north-star tolerance and are measurably
less accurate on the same inputs."""
import numpy as np
import pytest

from oracle import attn_oracle as ora
from oracle import inputs
from tests.gpu_util import assert_parity, to_dev

pytestmark = pytest.mark.gpu


def half_ulp(x):
    """Half the fp16 spacing at |x| (subnormal spacing 2^-24 below 2^-14)."""
    a = np.abs(x.astype(np.float32))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -14)))
    return 0.5 * np.exp2(e - 10)


def fp32_bound_ok(got, want):
    err = np.abs(got.astype(np.float32) - want)
    lim = np.maximum(half_ulp(want), half_ulp(got)) + 4e-6 * (1 + np.abs(want))
    return err, bool((err <= lim).all())


def normalised_qk(ex, case):
    """The case's q and k after the library's own RMSNorm (+ RoPE) kernels
    (animaxs_rmsnorm_heads_half / animaxs_rms_rope_split_half, the arithmetic
    of the fused prologue), as fp16 arrays: the attention of the fp32 mode is
    then compared with the fp32 oracle on exactly these inputs."""
    import torch
    if case.qk_norm == "none":
        return case.q, case.k
    res = []
    for x in (case.q, case.k):
        b, s, h, d = x.shape
        t = to_dev(x)
        o = torch.empty_like(t)
        st = torch.cuda.current_stream()
        if case.qk_norm == "rms_rope":
            ex.rms_rope_split_half(st, t, o, None, to_dev(case.rope_table), tokens=s, heads=h, head_dim=d)
        else:
            ex.rmsnorm_heads_half(st, t, o, None, tokens=s, heads=h, head_dim=d)
        torch.cuda.synchronize()
        res.append(o.cpu().numpy())
    return res


def oracle_on_normalised(ex, case):
    qn, kn = normalised_qk(ex, case)
    return ora.attention(qn, kn, case.v, causal=case.causal, kv_valid_len=case.kv_valid_len)


def _run(numerics, case, layout="token", **kw):
    import torch

    from animaxs_b200 import AttentionExecutor
    ex = AttentionExecutor(0, numerics=numerics)
    try:
        q, k, v = to_dev(case.q), to_dev(case.k), to_dev(case.v)
        if layout == "head":
            q, k, v = (t.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3) for t in (q, k, v))
        rope = None if case.rope_table is None else to_dev(case.rope_table)
        valid = None if case.kv_valid_len is None else case.kv_valid_len[0]
        out = ex.attention(q, k, v, causal=case.causal, qk_norm=case.qk_norm, rope_table=rope,
                           kv_valid_len=valid, **kw)
        torch.cuda.synchronize()
        ex.synchronize()
        return out.cpu().numpy()
    finally:
        ex.close()


@pytest.mark.parametrize("name", ["dit_self_1024", "qwen_causal_padded", "dit_cross_masked"])
def test_fp32_numerics_is_the_rounded_fp32_result(name):
    case = {"dit_self_1024": lambda: inputs.dit_self(seed=0, grid=(1, 32, 32)),
            "qwen_causal_padded": lambda: inputs.qwen_prefill(layer=3),
            "dit_cross_masked": lambda: inputs.dit_cross(seed=2, q_len=1024, kv_valid=128)}[name]()
    from animaxs_b200 import AttentionExecutor
    ex = AttentionExecutor(0)
    try:
        want = oracle_on_normalised(ex, case)
    finally:
        ex.close()
    layout = "head" if name.startswith("qwen") else "token"
    got32 = _run("fp32ScoresAndSoftmax", case, layout)
    err32, ok = fp32_bound_ok(got32, want)
    assert ok, f"{name}: fp32 numerics off the rounded fp32 result, worst {err32.max():.3e}"
    got16 = _run("legacy", case, layout)
    assert_parity(got16.astype(np.float32), case.oracle(), what=f"{name} legacy")
    err16 = np.abs(got16.astype(np.float32) - want)
    assert err32.mean() < err16.mean(), (name, float(err32.mean()), float(err16.mean()))
    assert err32.max() <= err16.max(), (name, float(err32.max()), float(err16.max()))


def test_fp32_numerics_head_dim_64_and_probe():
    """The adapter's head_dim 64, with the score probe on (its own kernel instantiation)."""
    import torch

    from animaxs_b200 import AttentionExecutor
    from animaxs_b200.probe import ScoreProbe
    case = inputs.adapter_attention(seed=4, target_tokens=512)
    ex = AttentionExecutor(0, numerics="fp32ScoresAndSoftmax")
    try:
        q, k, v = to_dev(case.q), to_dev(case.k), to_dev(case.v)
        probe = ScoreProbe(q.device)
        ex.set_score_probe(probe)
        out = ex.attention(q, k, v, qk_norm="rms_rope", rope_table=to_dev(case.rope_table))
        ex.set_score_probe(None)
        torch.cuda.synchronize()
        ex.synchronize()
        stats = probe.read()
        want = oracle_on_normalised(ex, case)
    finally:
        ex.close()
    err, ok = fp32_bound_ok(out.cpu().numpy(), want)
    assert ok, f"head_dim 64 fp32 numerics worst {err.max():.3e}"
    assert stats.flags == 0 and 0 < stats.max_abs < 100


def test_fp32_numerics_through_the_reference_call():
    """encode() on head-major buffers (the layout of the reference's encodeFP32)."""
    import torch

    from animaxs_b200 import AttentionExecutor
    case = inputs.qwen_prefill(layer=0, valid=None)
    ex = AttentionExecutor(0, numerics="fp32ScoresAndSoftmax")
    try:
        # plain attention (no fused norm): the reference's encode call shape, causal GQA
        qh = to_dev(case.q[0].transpose(1, 0, 2).copy())
        kh = to_dev(case.k[0].transpose(1, 0, 2).copy())
        vh = to_dev(case.v[0].transpose(1, 0, 2).copy())
        out = torch.empty_like(qh)
        ex.execute(qh, kh, vh, out, heads=16, query_count=512, key_count=512, head_dim=128,
                   key_value_heads=8, causal=True)
    finally:
        ex.close()
    want = ora.attention(case.q, case.k, case.v, causal=True)[0].transpose(1, 0, 2)
    err, ok = fp32_bound_ok(out.cpu().numpy(), want)
    assert ok, f"encode fp32 numerics worst {err.max():.3e}"
