"""CPU tests of the C ABI: the library loads, exports every function the header
declares, and its host-side logic (validation mirroring
AttentionExecutor.validate, RoPE tables, GQA map, scratch sizing) works
without a GPU."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from oracle import attn_oracle as ora
from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "animaxs_attn.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(animaxs_[a-z0-9_]+)\s*\(", text)))


def _header_abi_version():
    m = re.search(r"#define ANIMAXS_ATTN_ABI_VERSION (\d+)", open(HEADER).read())
    return int(m.group(1))


@pytest.fixture(scope="module")
def lib():
    from animaxs_b200 import _lib
    return _lib.lib()


def test_library_exports_every_declared_symbol(lib):
    from animaxs_b200 import _lib
    names = _declared()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (animaxs_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    # and the ctypes binding knows every one of them
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)
    assert lib.animaxs_attn_abi_version() == _lib.ABI_VERSION == _header_abi_version()


def test_library_links_no_nccl_or_cudart_at_load_time():
    from animaxs_b200 import _lib
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "libnccl" not in out and "libcudart" not in out


def test_create_fails_cleanly_without_gpu(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    ctx = ctypes.c_void_p()
    assert lib.animaxs_attn_create(0, ctypes.byref(ctx)) == -6  # ANIMAXS_ERR_NO_DEVICE
    assert not ctx.value


def _desc(lib, **kw):
    from animaxs_b200._lib import AttnDesc
    d = AttnDesc()
    lib.animaxs_attn_desc_init(ctypes.byref(d), kw.pop("batch", 1), kw.pop("heads", 16),
                               kw.pop("kv_heads", 16), kw.pop("q_len", 1024),
                               kw.pop("kv_len", 1024), kw.pop("head_dim", 128))
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def _validate(lib, d, ptrs=(0x1000, 0x2000, 0x3000, 0x4000)):
    return lib.animaxs_attn_validate(None, ctypes.byref(d), *[ctypes.c_void_p(p) for p in ptrs])


def test_validation_mirrors_reference(lib):
    ok = _desc(lib)
    assert _validate(lib, ok) == 0
    # shape rules (AttentionExecutor.swift:784-789)
    assert _validate(lib, _desc(lib, heads=6, kv_heads=4)) == -1
    assert _validate(lib, _desc(lib, q_len=0)) == -1
    assert _validate(lib, _desc(lib, causal=1, q_len=100, kv_len=200)) == -1
    assert _validate(lib, _desc(lib, causal=1, q_len=100, kv_len=100)) == 0
    # head dims: 128 (DiT, Qwen) and 64 (LLM adapter) run; others are unsupported
    assert _validate(lib, _desc(lib, head_dim=64)) == 0
    assert _validate(lib, _desc(lib, head_dim=96)) == -2
    assert _validate(lib, _desc(lib, head_dim=32)) == -2
    # VAE middle attention: one head of 384 (VAEDecoder.swift:351-410); 256 shares its kernel.
    assert _validate(lib, _desc(lib, heads=1, kv_heads=1, head_dim=384)) == 0
    assert _validate(lib, _desc(lib, head_dim=256)) == 0
    assert _validate(lib, _desc(lib, head_dim=512)) == -2
    assert _validate(lib, _desc(lib, head_dim=384, qk_norm=1)) == -2  # fused norm: 64 / 128 only
    # null and misaligned buffers, misaligned stride
    assert _validate(lib, ok, (0, 0x2000, 0x3000, 0x4000)) == -1
    assert _validate(lib, ok, (0x1008, 0x2000, 0x3000, 0x4000)) == -1
    assert _validate(lib, _desc(lib, q_tok_stride=2047 * 1)) == -1
    # buffer range (:808-823): q needs 1024*2048*2 bytes
    assert _validate(lib, _desc(lib, q_bytes=1024 * 2048 * 2)) == 0
    assert _validate(lib, _desc(lib, q_bytes=1024 * 2048 * 2 - 2)) == -3
    # masks, scale, rope
    assert _validate(lib, _desc(lib, kv_valid_len=1025)) == -1
    assert _validate(lib, _desc(lib, kv_valid_len=-1)) == -1
    assert _validate(lib, _desc(lib, scale=-1.0)) == -1
    # normalisation targets (q and k / q only / k only)
    for t in (0, 1, 2):
        assert _validate(lib, _desc(lib, qk_norm_targets=t)) == 0
    assert _validate(lib, _desc(lib, qk_norm_targets=3)) == -1
    assert _validate(lib, _desc(lib, qk_norm=2)) == -1            # rope table missing
    assert _validate(lib, _desc(lib, qk_norm=2, rope_table=0x5000, rope_rows=1023)) == -1
    assert _validate(lib, _desc(lib, qk_norm=2, rope_table=0x5000, rope_rows=1024)) == 0
    assert _validate(lib, _desc(lib, qk_norm=7)) == -1
    # overflow
    assert _validate(lib, _desc(lib, q_batch_stride=1 << 45, batch=2)) == -8
    # numerics (AttentionExecutor.init numerics:): legacy and fp32ScoresAndSoftmax run at
    # head_dim 64 / 128; bf16Compute is not built; fp32 on the wide-head kernel is not built
    assert _validate(lib, _desc(lib, numerics=1)) == 0
    assert _validate(lib, _desc(lib, numerics=1, head_dim=64)) == 0
    assert _validate(lib, _desc(lib, numerics=2)) == -2
    assert _validate(lib, _desc(lib, numerics=3)) == -1
    assert _validate(lib, _desc(lib, numerics=1, heads=1, kv_heads=1, head_dim=384)) == -2


def test_scratch_bytes(lib):
    d = _desc(lib, qk_norm=1, q_len=4096, kv_len=512)
    n = ctypes.c_int64()
    assert lib.animaxs_attn_scratch_bytes(ctypes.byref(d), ctypes.byref(n)) == 0
    assert n.value == 4096 * 16 * 256 + 512 * 16 * 256
    # only the copies the prologue writes: q only (k cached by the caller), k only
    d.qk_norm_targets = 1
    lib.animaxs_attn_scratch_bytes(ctypes.byref(d), ctypes.byref(n))
    assert n.value == 4096 * 16 * 256
    d.qk_norm_targets = 2
    lib.animaxs_attn_scratch_bytes(ctypes.byref(d), ctypes.byref(n))
    assert n.value == 512 * 16 * 256
    d.qk_norm = 0
    lib.animaxs_attn_scratch_bytes(ctypes.byref(d), ctypes.byref(n))
    assert n.value == 0


def test_cache_and_streamer_need_a_context(lib):
    """The cross-K/V cache and weight streamer entry points reject a missing
    context / handle before touching a device."""
    h = ctypes.c_void_p()
    assert lib.animaxs_cross_kv_cache_create(None, 28, 1, 512, 16, 128, None, 0, ctypes.byref(h)) == -1
    assert lib.animaxs_weight_streamer_create(None, 1024, 2, ctypes.byref(h)) == -1
    assert lib.animaxs_weight_streamer_slot(None, 0) is None
    assert lib.animaxs_cross_kv_cache_reset(None) == -1
    n = ctypes.c_int64()
    assert lib.animaxs_cross_kv_cache_bytes(28, 1, 512, 16, 128, ctypes.byref(n)) == 0
    assert n.value == 28 * 512 * 2 * 2048 * 2      # CrossKVCache: 28 x 4 MiB
    assert lib.animaxs_cross_kv_cache_bytes(28, 1, 512, 16, 96, ctypes.byref(n)) == -2


def test_noalloc_status_without_gpu(lib):
    """The no-alloc status query fails cleanly without a device (it never allocates)."""
    assert lib.animaxs_attn_noalloc_status() in (-6, -4)


@pytest.mark.parametrize("grid", [(1, 32, 32), (1, 64, 64), (2, 8, 12)])
def test_rope3d_table_helper(grid):
    from animaxs_b200 import DitRoPE
    got = DitRoPE.generate(*grid).reshape(-1, 64, 2, 2)
    np.testing.assert_allclose(got, ora.dit_rope_table(*grid), atol=3e-6)


def test_rope1d_table_helper():
    from animaxs_b200 import qwen_rope
    got = qwen_rope(512).reshape(512, 64, 2, 2)
    np.testing.assert_allclose(got, ora.rope1d_table(512, 1e6), atol=4e-5)


def test_adapter_rope_table_helper():
    """LLMAdapterMetal.makeRope (LLMAdapterMetal.swift:162-178) through the C
    helper: [tokens][32][2][2], theta 1e4, 64-wide heads."""
    from animaxs_b200 import adapter_rope
    got = adapter_rope(512).reshape(512, 32, 2, 2)
    ref = ora.adapter_rope_table(512)
    np.testing.assert_allclose(got, ref, atol=4e-5)
    # token 1, pair 0: angle 1 rad; pair 16: 1 / 10000^(32/64) = 0.01 rad
    np.testing.assert_allclose(got[1, 0].ravel(), [np.cos(1.0), -np.sin(1.0), np.sin(1.0), np.cos(1.0)],
                               atol=1e-6)
    np.testing.assert_allclose(got[1, 16, 1, 0], np.sin(0.01), atol=1e-7)


def test_gqa_helper():
    from animaxs_b200 import AttentionValidationError, GqaHeadMapping
    assert [GqaHeadMapping.kv_head(h, 16, 8) for h in range(16)] == [ora.gqa_kv_head(h, 16, 8) for h in range(16)]
    with pytest.raises(AttentionValidationError):
        GqaHeadMapping.kv_head(0, 6, 4)


def test_executor_mirror_errors_without_gpu():
    """The Python mirror raises the reference's validation messages before any GPU work."""
    from animaxs_b200 import AttentionExecutor, AttentionInputLayout, AttentionValidationError
    ex = AttentionExecutor.__new__(AttentionExecutor)
    from animaxs_b200 import _lib
    ex._lib = _lib.lib()
    ex.layout = AttentionInputLayout.head_major
    ex.numerics = "legacy"
    ex.tile_rows = 128
    with pytest.raises(AttentionValidationError, match="keyValueHeads == heads"):
        ex.make_desc(heads=2, query_count=4, key_count=4, head_dim=64, key_value_heads=1,
                     layout=AttentionInputLayout.token_major(128))
    assert ex.maximum_score_scratch_bytes(1024) == 128 * 1024 * 2
    assert ex.maximum_score_scratch_bytes(37, 19) == 19 * 37 * 2
    ex.numerics = "fp32ScoresAndSoftmax"
    assert ex.maximum_score_scratch_bytes(37, 19) == 19 * 37 * 4
    with pytest.raises(AttentionValidationError, match="token-major"):
        ex.make_desc(heads=2, query_count=4, key_count=4, head_dim=64,
                     layout=AttentionInputLayout.token_major(128))


def _pdesc(lib, m=256, n=768, k=256, epilogue=1, **kw):
    from animaxs_b200._lib import ProjDesc
    d = ProjDesc()
    assert lib.animaxs_proj_desc_init(ctypes.byref(d), m, n, k, epilogue) == 0
    if epilogue == 1:
        d.qk_norm, d.q_cols, d.k_cols = 1, 256, 256
    if epilogue == 2:
        d.gate = 0x6000
    for key, val in kw.items():
        setattr(d, key, val)
    return d


def _pvalidate(lib, d, ptrs=(0x1000, 0x2000, 0x3000)):
    return lib.animaxs_proj_validate(None, ctypes.byref(d), *[ctypes.c_void_p(p) for p in ptrs])


def test_projection_validation(lib):
    """animaxs_proj_validate: shapes, alignment, head multiples, epilogue inputs."""
    assert _pvalidate(lib, _pdesc(lib)) == 0
    assert _pvalidate(lib, _pdesc(lib, epilogue=0)) == 0
    assert _pvalidate(lib, _pdesc(lib, epilogue=2, n=256)) == 0
    assert _pvalidate(lib, _pdesc(lib, m=0)) == -1
    assert _pvalidate(lib, _pdesc(lib, k=100)) == -1                    # k % 8
    assert _pvalidate(lib, _pdesc(lib), (0x1008, 0x2000, 0x3000)) == -1  # alignment
    assert _pvalidate(lib, _pdesc(lib, x_stride=128)) == -1             # stride < k
    assert _pvalidate(lib, _pdesc(lib, epilogue=3)) == -1
    assert _pvalidate(lib, _pdesc(lib, q_cols=192)) == -2               # heads of 128
    assert _pvalidate(lib, _pdesc(lib, q_cols=512, k_cols=512)) == -2   # q + k > n
    assert _pvalidate(lib, _pdesc(lib, qk_norm=0)) == -1
    assert _pvalidate(lib, _pdesc(lib, qk_norm=2)) == -1                # rope table missing
    assert _pvalidate(lib, _pdesc(lib, qk_norm=2, rope_table=0x5000, rope_rows=256)) == 0
    assert _pvalidate(lib, _pdesc(lib, qk_norm=2, rope_table=0x5000, rope_rows=255)) == -1
    assert _pvalidate(lib, _pdesc(lib, epilogue=2, n=256, gate=None)) == -1
    assert _pvalidate(lib, _pdesc(lib, epilogue=2, n=256, out_stride=258)) == -1  # fp32 rows: 16 B


def test_projection_quantized_weight_validation(lib):
    """W8/W4 weight storage: scale/zero present and 2-byte aligned, packed rows
    wide enough (ceil(k / 2) bytes for W4, k for W8); the packed codes need no
    16-byte alignment (they are decoded into an aligned copy first)."""
    from animaxs_b200._lib import WEIGHT_W4, WEIGHT_W8
    q = dict(w_scale=0x7000, w_zero=0x8000)
    assert _pvalidate(lib, _pdesc(lib, w_storage=WEIGHT_W4, w_packed_stride=128, **q)) == 0
    assert _pvalidate(lib, _pdesc(lib, w_storage=WEIGHT_W8, w_packed_stride=256, **q)) == 0
    assert _pvalidate(lib, _pdesc(lib, w_storage=WEIGHT_W4, w_packed_stride=128, **q),
                      (0x1000, 0x2003, 0x3000)) == 0                    # byte-aligned codes
    assert _pvalidate(lib, _pdesc(lib, w_storage=WEIGHT_W4, w_packed_stride=127, **q)) == -1
    assert _pvalidate(lib, _pdesc(lib, w_storage=WEIGHT_W8, w_packed_stride=128, **q)) == -1
    assert _pvalidate(lib, _pdesc(lib, w_storage=WEIGHT_W4, w_packed_stride=128, w_scale=0x7000)) == -1
    assert _pvalidate(lib, _pdesc(lib, w_storage=WEIGHT_W4, w_packed_stride=128, w_scale=0x7001,
                                  w_zero=0x8000)) == -1
    assert _pvalidate(lib, _pdesc(lib, w_storage=3, w_packed_stride=256, **q)) == -1
    assert _pvalidate(lib, _pdesc(lib), (0x1000, 0x2003, 0x3000)) == -1   # fp16 weight: 16 B


def test_dequant_requires_context(lib):
    """animaxs_dequant_to_half refuses a null context before touching a device."""
    assert lib.animaxs_dequant_to_half(None, 4, 0x1000, 0x2000, 0x3000, 0x4000, 4, 64, 32, 64, None) == -1


def test_peer_group_rejects_bad_arguments(lib):
    """The fused head-sharded entry points check their arguments before any
    device call."""
    grp = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    assert lib.animaxs_peer_group_create(None, 2, 0, 1024, ctypes.byref(grp), h) == -1
    assert lib.animaxs_peer_group_connect(None, h) == -1
    assert lib.animaxs_peer_group_output(None) is None
    assert lib.animaxs_peer_group_destroy(None) == 0
    assert lib.animaxs_attn_forward_head_sharded_peer(None, None, None, 0, 0, 0, 0, None) == -1


def test_header_compiles_as_c11_and_cxx17(tmp_path):
    """The header is consumed by C (and a Swift module map): it must compile as
    strict C11 as well as C++17, with every declaration usable."""
    src = tmp_path / "use.c"
    src.write_text(
        '#include "animaxs_attn.h"\n'
        "int main(void) {\n"
        "  animaxs_attn_desc d; animaxs_proj_desc p; unsigned int stats[4];\n"
        "  (void)animaxs_attn_desc_init(&d, 1, 16, 16, 4096, 4096, 128);\n"
        "  (void)animaxs_proj_desc_init(&p, 256, 768, 256, ANIMAXS_PROJ_QKV_NORM);\n"
        "  p.w_storage = ANIMAXS_WEIGHT_W4;\n"
        "  (void)animaxs_attn_set_score_probe((animaxs_attn_ctx*)0, stats);\n"
        "  animaxs_peer_group* g = (animaxs_peer_group*)0; (void)animaxs_peer_group_output(g);\n"
        "  return ANIMAXS_ATTN_ABI_VERSION == 2 && ANIMAXS_PROBE_NAN == 1u ? 0 : 1;\n"
        "}\n")
    inc = os.path.dirname(HEADER)
    for cmd in (["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-fsyntax-only"],
                ["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-x", "c++"]):
        res = subprocess.run([*cmd, "-I", inc, str(src)], capture_output=True, text=True)
        assert res.returncode == 0, res.stderr


def test_score_probe_requires_context(lib):
    assert lib.animaxs_attn_set_score_probe(None, None) == -1


def test_probe_stats_decoding_follows_the_reference():
    """NumericalMonitor.Stats (NumericalMonitor.swift:136-161): flag bits,
    max |score| from its float bits, condition wording and precedence."""
    from animaxs_b200.probe import ProbeStats
    assert ProbeStats.from_words([0, 0, 0xFFFFFFFF, 0]) == ProbeStats()
    assert not ProbeStats().has_issue
    st = ProbeStats.from_words([8 | 2, 0x47CA0000, 42, 0])
    assert st.has_half_overflow and st.has_pos_inf and st.first_index == 42
    assert st.max_abs == 103424.0
    assert st.condition == "positive Inf detected"
    assert ProbeStats(flags=1 | 4).condition == "NaN detected"
    assert ProbeStats(flags=4).condition == "negative Inf detected"
    assert ProbeStats(flags=8).condition == "value exceeded FP16 finite range"
    import re
    h = open(HEADER).read()
    got = {n: int(v) for n, v in re.findall(r"#define ANIMAXS_PROBE_(\w+) (\d+)u", h)}
    assert got == {"NAN": 1, "POS_INF": 2, "NEG_INF": 4, "HALF_OVERFLOW": 8}


def test_selftest_rejects_bad_timeout(lib):
    """The failure-detection self-test validates its limit before touching a device."""
    assert lib.animaxs_attn_selftest_wait_timeout(None, 1000, None) == -1
