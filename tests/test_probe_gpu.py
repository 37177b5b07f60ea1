"""GPU tests of the attention score-health probe (``animaxs_attn_set_score_probe``),
the counterpart of the reference's NumericalMonitor score probes
(attention_softmax_rows_probe, AnimaKernels.metal:1738-1830).

Flags and the first flagged key are exact.  The recorded max |score| is an
fp32 score computed in a different summation order than the oracle's, so it
is compared to 1e-3 relative.
"""
import numpy as np
import pytest

from oracle import attn_oracle as ora
from oracle import inputs
from tests.gpu_util import to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ex():
    from animaxs_b200 import AttentionExecutor
    e = AttentionExecutor(0)
    yield e
    e.close()


def _probe():
    from animaxs_b200 import ScoreProbe
    return ScoreProbe("cuda")


def _run(ex, probe, q, k, v, **kw):
    import torch
    ex.set_score_probe(probe)
    try:
        out = ex.attention(to_dev(q), to_dev(k), to_dev(v), **kw)
    finally:
        ex.set_score_probe(None)
    ex.synchronize()
    torch.cuda.synchronize()
    return out, probe.read()


def test_healthy_dit_self_attention_records_max_score(ex):
    """1024-token DiT self-attention with fused RMSNorm + RoPE: no flag; the
    magnitude is the largest scaled score of the normalised q/k."""
    case = inputs.dit_self(seed=3, grid=(1, 32, 32), heads=16)
    pr = _probe()
    _, st = _run(ex, pr, case.q, case.k, case.v, qk_norm="rms_rope", rope_table=to_dev(case.rope_table))
    qn = ora.apply_split_half_rope(ora.rms_norm_heads(case.q), case.rope_table)
    kn = ora.apply_split_half_rope(ora.rms_norm_heads(case.k), case.rope_table)
    flags, mx, first = ora.score_health(ora.to_fp16_storage(qn), ora.to_fp16_storage(kn))
    assert st.flags == flags == 0 and st.first_index == first == 0xFFFFFFFF
    assert st.max_abs == pytest.approx(mx, rel=1e-3)


def test_nan_key_is_flagged_with_its_index(ex):
    q, k, v = inputs.draw_qkv(5, (1, 300, 4, 128), (1, 300, 4, 128))
    k = k.copy()
    k[0, 37, 2, 5] = np.nan
    pr = _probe()
    _, st = _run(ex, pr, q, k, v)
    flags, mx, first = ora.score_health(q, k)
    assert st.has_nan and st.flags == flags and st.first_index == first == 37
    assert st.condition == "NaN detected"
    assert st.max_abs == pytest.approx(mx, rel=1e-3)


def test_infinite_scores_and_half_overflow(ex):
    """+Inf and -Inf keys (strictly positive q) and a finite score beyond the
    fp16 range, each flagged; the magnitude covers only finite scores."""
    rng = np.random.default_rng(7)
    q = (np.abs(rng.standard_normal((1, 256, 2, 128))) + 0.1).astype(np.float16)
    k = rng.standard_normal((1, 256, 2, 128)).astype(np.float16)
    v = rng.standard_normal((1, 256, 2, 128)).astype(np.float16)
    k[0, 9, 0, :] = np.inf
    k[0, 11, 1, :] = -np.inf
    k[0, 200, 0, :] = 60.0    # q.k ~ 128 * 0.9 * 60 -> ~6e3 * 1/sqrt(128) ... made large below
    q[0, 100, 0, :] = 200.0   # row 100 x key 200: 128 * 200 * 60 / sqrt(128) = 1.36e5 > 65504
    pr = _probe()
    _, st = _run(ex, pr, q, k, v)
    flags, mx, first = ora.score_health(q, k)
    assert flags == 2 | 4 | 8
    assert st.flags == flags and st.first_index == first == 9
    assert st.has_pos_inf and st.has_neg_inf and st.has_half_overflow
    assert st.condition == "positive Inf detected"
    assert st.max_abs == pytest.approx(mx, rel=1e-3) and st.max_abs > 65504


def test_masked_keys_are_not_probed(ex):
    """A NaN behind the key padding is not seen; behind the causal mask it is
    seen only by the rows that attend to it."""
    q, k, v = inputs.draw_qkv(9, (1, 512, 2, 128), (1, 512, 2, 128))
    k = k.copy()
    k[0, 400, 1, 0] = np.nan
    pr = _probe()
    _, st = _run(ex, pr, q, k, v, kv_valid_len=300)
    assert st.flags == 0 and st.first_index == 0xFFFFFFFF
    flags, mx, _ = ora.score_health(q, k, kv_valid_len=300)
    assert st.max_abs == pytest.approx(mx, rel=1e-3)
    pr.reset()
    _, st = _run(ex, pr, q, k, v, causal=True)
    flags, mx, first = ora.score_health(q, k, causal=True)
    assert st.flags == flags == 1 and st.first_index == first == 400


def test_encode_probe_argument_accumulates_and_is_released(ex):
    """The reference's encode(probe:) form: the slot accumulates over calls
    (flags OR, max, min index) and a call without a probe leaves it alone."""
    import torch
    from animaxs_b200 import AttentionInputLayout
    q, k, v = inputs.draw_qkv(11, (1, 128, 2, 128), (1, 128, 2, 128))
    k = k.copy()
    k[0, 70, 0, 3] = np.nan
    pr = _probe()
    s = torch.cuda.current_stream()
    lay = AttentionInputLayout.token_major(256)
    o = torch.empty(1, 128, 2, 128, dtype=torch.float16, device="cuda")
    ex.encode(s, to_dev(q), to_dev(k), to_dev(v), o, heads=2, query_count=128, key_count=128, head_dim=128,
              layout=lay, probe=pr)
    k2 = k.copy()
    k2[0, 70, 0, 3] = 0.0
    k2[0, 20, 1, 0] = np.inf
    ex.encode(s, to_dev(q), to_dev(k2), to_dev(v), o, heads=2, query_count=128, key_count=128, head_dim=128,
              layout=lay, probe=pr)
    ex.synchronize(s)
    st = pr.read()
    assert st.has_nan and st.first_index == 20 and (st.has_pos_inf or st.has_neg_inf)
    before = pr.words.clone()
    ex.encode(s, to_dev(q), to_dev(k), to_dev(v), o, heads=2, query_count=128, key_count=128, head_dim=128,
              layout=lay)
    ex.synchronize(s)
    assert torch.equal(pr.words, before)


def test_probe_with_wide_heads_is_rejected(ex):
    from animaxs_b200 import AttentionValidationError
    q, k, v = inputs.draw_qkv(1, (1, 128, 1, 384), (1, 128, 1, 384))
    pr = _probe()
    ex.set_score_probe(pr)
    try:
        with pytest.raises(AttentionValidationError):
            ex.attention(to_dev(q), to_dev(k), to_dev(v))
    finally:
        ex.set_score_probe(None)
    ex.attention(to_dev(q), to_dev(k), to_dev(v))   # without the probe it runs
    ex.synchronize()
