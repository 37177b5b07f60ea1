"""Pin the CPU oracle (oracle/attn_oracle.py) against fixtures produced by the
reference's own PyTorch oracles (tests/golden/make_golden.py) and against the
reference's Swift known-answer tests (DitRoPETests, DiTBlockTests,
GqaHeadMappingTests)."""
import os

import numpy as np
import pytest

from oracle import attn_oracle as ora
from oracle import inputs
from tests.conftest import GOLDEN


def _npz(name):
    return np.load(os.path.join(GOLDEN, name))


def _checksum(x):
    x = np.asarray(x, dtype=np.float64)
    return np.array([x.sum(), np.abs(x).sum(), (x * x).sum()])


@pytest.mark.parametrize("grid", [(1, 32, 32), (1, 64, 64), (1, 128, 128)])
def test_rope3d_table_matches_reference(grid):
    g = _npz("rope_tables.npz")
    key = "rope3d_{}x{}x{}".format(*grid)
    tab = ora.dit_rope_table(*grid)
    rows = g[key + "_rows"]
    np.testing.assert_allclose(tab[rows], g[key + "_sample"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(_checksum(tab), g[key + "_checksum"], rtol=1e-6)


def test_rope3d_matches_reference_committed_golden():
    # scripts/oracle_out/dit_rope_oracle.npz (the reference's own fixture)
    g = _npz("rope_tables.npz")
    tab = ora.dit_rope_table(1, 32, 32)
    np.testing.assert_allclose(tab[g["committed_rope_rows"]], g["committed_rope_sample"], atol=2e-6)
    np.testing.assert_allclose(_checksum(tab), g["committed_rope_checksum"], rtol=1e-6)


def test_rope1d_matches_reference():
    g = _npz("rope_tables.npz")
    tab = ora.rope1d_table(512, 1.0e6)
    rows = g["rope1d_512_rows"]
    # Angles reach 511 rad, where one fp32 ulp of the inverse frequency (torch's
    # pow vs libm powf, which the Swift makeRope uses) moves cos/sin by ~3e-5.
    tol = 4e-5
    np.testing.assert_allclose(tab[rows, :, 0, 0], g["rope1d_512_cos"], atol=tol)
    np.testing.assert_allclose(tab[rows, :, 1, 0], g["rope1d_512_sin"], atol=tol)
    # precompute_freqs_cis returns -sin for the second half; the table stores it at [0,1]
    np.testing.assert_allclose(tab[rows, :, 0, 1], g["rope1d_512_nsin"], atol=tol)


def test_rope3d_known_answers():
    # DitRoPETests.swift: token 0 is the identity; w=1 / w=17 anchors; t,h,w order.
    tab = ora.dit_rope_table(1, 32, 32)
    np.testing.assert_allclose(tab[0].reshape(64, 4), np.tile([1, 0, 0, 1], (64, 1)), atol=1e-7)
    np.testing.assert_allclose(tab[1, 43].ravel(), [np.cos(1.0), -np.sin(1.0), np.sin(1.0), np.cos(1.0)], atol=1e-6)
    np.testing.assert_allclose(tab[17, 43].ravel(), [np.cos(17.0), -np.sin(17.0), np.sin(17.0), np.cos(17.0)], atol=1e-5)
    # h=1 (token 32): first height pair (index 22) rotates by 1 rad, width pairs are identity
    np.testing.assert_allclose(tab[32, 22].ravel(), [np.cos(1.0), -np.sin(1.0), np.sin(1.0), np.cos(1.0)], atol=1e-6)
    np.testing.assert_allclose(tab[32, 43:].reshape(-1, 4), np.tile([1, 0, 0, 1], (21, 1)), atol=1e-7)
    # thetas (DitRoPETests.swift:114-120)
    assert abs(float(np.float32(10000.0 * 4.0 ** (42 / 40))) - 42870.938501451725) < 0.01


def test_split_half_pairing_known_answers():
    # DiTBlockTests.swift:18-65: pairs (p, p+D/2), not adjacent.
    x = np.array([1, 2, 3, 4], np.float32).reshape(1, 1, 1, 4)
    table = np.zeros((1, 2, 2, 2), np.float32)
    table[0, 0] = [[0, -1], [1, 0]]     # 90 degrees
    table[0, 1] = [[-1, 0], [0, -1]]    # 180 degrees
    out = ora.apply_split_half_rope(x, table).ravel()
    np.testing.assert_allclose(out, [-3, -2, 1, -4], atol=1e-6)
    x8 = np.array([1, 2, 3, 4, 10, 20, 30, 40], np.float32).reshape(1, 1, 1, 8)
    ident = np.zeros((1, 4, 2, 2), np.float32)
    ident[0, :, 0, 0] = 1
    ident[0, :, 1, 1] = 1
    np.testing.assert_allclose(ora.apply_split_half_rope(x8, ident), x8)


def test_gqa_mapping_table():
    # GqaHeadMappingTests.swift:23-43
    assert [ora.gqa_kv_head(h, 16, 8) for h in range(16)] == [0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6, 6, 7, 7]
    assert [ora.gqa_kv_head(h, 32, 8) for h in (0, 7, 8, 31)] == [0, 1, 2, 7]
    with pytest.raises(ValueError):
        ora.gqa_kv_head(0, 6, 4)


def test_rms_norm_shared_weight():
    # DiTBlockTests.swift:89-115: per-head RMSNorm with a shared [D] weight
    x = np.arange(16, dtype=np.float32).reshape(1, 1, 2, 8) - 5
    w = np.linspace(0.5, 2, 8).astype(np.float32)
    out = ora.rms_norm_heads(x, w)
    for h in range(2):
        row = x[0, 0, h]
        np.testing.assert_allclose(out[0, 0, h], row / np.sqrt(np.mean(row * row) + 1e-6) * w, rtol=1e-6)


SMALL = {
    "dit_self_256": lambda: inputs.dit_self(seed=10, grid=(1, 16, 16), heads=2),
    "dit_cross_192x96_valid40": lambda: inputs.dit_cross(seed=11, q_len=192, kv_len=96, heads=2, kv_valid=40),
    "dit_cross_130x200": lambda: inputs.dit_cross(seed=12, q_len=130, kv_len=200, heads=2, kv_valid=None),
    "qwen_160_h4kv2_valid100": lambda: inputs.qwen_prefill(layer=0, seq_len=160, heads=4, kv_heads=2, valid=100),
}


@pytest.mark.parametrize("name", sorted(SMALL))
def test_oracle_matches_reference_small(name):
    g = _npz("attn_small.npz")
    case = SMALL[name]()
    got_in = np.concatenate([_checksum(case.q), _checksum(case.k), _checksum(case.v)])
    np.testing.assert_allclose(got_in, g[name + "_in_checksum"], rtol=1e-9)
    out = case.oracle()
    np.testing.assert_allclose(out, g[name + "_out"], atol=2e-5, rtol=0)


def _cfg_cases():
    out = {
        "cfg1": lambda: inputs.dit_self(seed=0, grid=(1, 32, 32)),
        "cfg2_masked": lambda: inputs.dit_cross(seed=0),
        "cfg2_unmasked": lambda: inputs.dit_cross(seed=0, kv_valid=None),
        "cfg3_l0": lambda: inputs.qwen_prefill(layer=0),
        "cfg3_l27": lambda: inputs.qwen_prefill(layer=27),
    }
    for p in (0, 7):
        for s in (0, 7):
            for b in (0, 27):
                tag = f"cfg4_p{p}_s{s}_b{b}"
                out[tag + "_self"] = (lambda p=p, s=s, b=b: inputs.workload_block(p, s, b)[0])
                out[tag + "_cross"] = (lambda p=p, s=s, b=b: inputs.workload_block(p, s, b)[1])
    out["cfg5"] = lambda: inputs.dit_self(seed=0, grid=(1, 128, 128))
    return out


CFG = _cfg_cases()
FAST_CFG = ["cfg1", "cfg2_masked", "cfg2_unmasked", "cfg3_l0", "cfg3_l27",
            "cfg4_p0_s0_b0_self", "cfg4_p7_s7_b27_cross", "cfg5"]


@pytest.mark.parametrize("name", FAST_CFG)
def test_oracle_matches_reference_configs(name):
    g = _npz("attn_configs.npz")
    case = CFG[name]()
    rows = g[name + "_rows"]
    got_in = np.concatenate([_checksum(case.q), _checksum(case.k), _checksum(case.v)])
    np.testing.assert_allclose(got_in, g[name + "_in_checksum"], rtol=1e-9)
    out = case.oracle(rows=rows)
    np.testing.assert_allclose(out, g[name + "_out"], atol=3e-5, rtol=0)


# ------------------------------------------------ fused projections (row f) --
def test_projection_oracle_matches_reference():
    """qkv_norm_projection / gate_add_projection against the reference's own
    linear + rms_norm + dit_rope + apply_split_half_rope and its gated residual
    update (tests/golden/proj_small.npz)."""
    g = _npz("proj_small.npz")
    seed, images, tokens, k, qh, kh, vc = (int(v) for v in g["qkv_meta"])
    x, w, qw, kw = inputs.proj_qkv(seed, images=images, tokens=tokens, k=k, q_heads=qh, k_heads=kh, v_cols=vc)
    np.testing.assert_allclose(np.concatenate([_checksum(x), _checksum(w), _checksum(qw), _checksum(kw)]),
                               g["qkv_in_checksum"], rtol=1e-12)
    table = ora.dit_rope_table(1, 8, 8)
    for mode, key in (("rms_rope", "qkv_rope_out"), ("rms", "qkv_rms_out")):
        got = ora.qkv_norm_projection(x, w, q_cols=qh * 128, k_cols=kh * 128, qk_norm=mode,
                                      q_norm_weight=qw, k_norm_weight=kw, rope_table=table, tokens=tokens)
        np.testing.assert_allclose(got, g[key], atol=2e-5, rtol=1e-5, err_msg=mode)
    seed, images, tokens, k, n = (int(v) for v in g["gate_meta"])
    xg, wg, res, gate = inputs.proj_gate(seed, images=images, tokens=tokens, k=k, n=n)
    np.testing.assert_allclose(np.concatenate([_checksum(xg), _checksum(wg), _checksum(res), _checksum(gate)]),
                               g["gate_in_checksum"], rtol=1e-12)
    got = ora.gate_add_projection(res, xg, wg, gate, tokens=tokens)
    np.testing.assert_allclose(got, g["gate_out"], atol=2e-5, rtol=1e-5)


def test_quant_decode_oracle_matches_reference():
    """dequant_to_half against the reference's own W8/W4 decoders on weights
    packed by its own quantizer (tests/golden/quant_small.npz): bit-exact fp16,
    and equal to the reference's fp32 reconstruction before the fp16 rounding;
    then a projection through the decoded W4 weight against the reference's
    linear (fp16 output, one fp16 ulp for the fp32 summation order)."""
    g = _npz("quant_small.npz")
    for name in ("w8", "w4", "w4opt", "w4wide"):
        bits, rows, k, _opt, _seed = (int(v) for v in g[name + "_meta"])
        got = ora.dequant_to_half(g[name + "_packed"], g[name + "_scale"], g[name + "_zero"], bits=bits, k=k)
        assert got.shape == (rows, k)
        assert np.array_equal(got.view(np.uint16), g[name + "_decoded_half"].view(np.uint16)), name
        assert np.array_equal(got, g[name + "_decoded_f32"].astype(np.float16)), name
    seed, m, k = (int(v) for v in g["proj_w4_meta"])
    y = ora.linear_fp16(inputs.proj_x(seed, m, k), g["w4wide_decoded_half"])
    np.testing.assert_allclose(y, g["proj_w4_out"], atol=2e-3, rtol=2e-3)


def test_quant_decode_oracle_layout():
    """Nibble order and group restart, on hand-made codes: byte 0x21 holds
    column 0 = 1 (low nibble) and column 1 = 2; column 64 uses the second
    group's scale and zero."""
    packed = np.zeros((1, 33), dtype=np.uint8)
    packed[0, 0] = 0x21
    packed[0, 32] = 0x03
    scale = np.array([[1.0, 0.5]], dtype=np.float16)
    zero = np.array([[0.0, 10.0]], dtype=np.float16)
    out = ora.dequant_to_half(packed, scale, zero, bits=4, k=65)
    assert out[0, 0] == 1 and out[0, 1] == 2 and out[0, 2] == 0
    assert out[0, 64] == np.float16(11.5)
    w8 = ora.dequant_to_half(np.array([[255, 7]], dtype=np.uint8), np.array([[0.25]], dtype=np.float16),
                             np.array([[-1.0]], dtype=np.float16), bits=8, k=2)
    assert w8[0, 0] == np.float16(62.75) and w8[0, 1] == np.float16(0.75)


def test_score_health_oracle():
    """score_health on planted values: flags, magnitude over finite scores,
    first flagged key, masks (key padding and causal) excluded."""
    rng = np.random.default_rng(0)
    q = (np.abs(rng.standard_normal((1, 8, 2, 64))) + 0.1).astype(np.float16)
    k = rng.standard_normal((1, 8, 2, 64)).astype(np.float16)
    flags, mx, first = ora.score_health(q, k)
    assert flags == 0 and first == 0xFFFFFFFF and mx > 0
    k2 = k.copy()
    k2[0, 5, 1, :] = np.inf
    k2[0, 6, 0, :] = -np.inf
    assert ora.score_health(q, k2) == (ora.PROBE_POS_INF | ora.PROBE_NEG_INF, mx, 5)
    k3 = k.copy()
    k3[0, 3, 0, 0] = np.nan
    assert ora.score_health(q, k3)[0::2] == (ora.PROBE_NAN, 3)
    assert ora.score_health(q, k3, kv_valid_len=3)[0::2] == (0, 0xFFFFFFFF)
    assert ora.score_health(q, k3, causal=True)[0::2] == (ora.PROBE_NAN, 3)
