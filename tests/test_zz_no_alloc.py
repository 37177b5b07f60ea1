"""GPU test of animaxs_attn_forward_noalloc, the allocation-free entry point.

Who needs it: callers that must not have device memory allocated for them --
an application that reserves the GPU's memory up front and treats any later
cudaMalloc as a failure, a host runtime whose own allocator must own every
device allocation, or a latency-critical loop where an allocation (which can
synchronise the device) is unacceptable.  The entry point keeps the fused
prologue's normalised q/k in a fixed 32 MiB device array instead.

The test calls it through the C ABI several times in a row (different shapes,
values and normalisation modes, so stale contents of the shared array would
show) and requires each output to be BIT-IDENTICAL to the allocating entry
point animaxs_attn_forward on the same inputs: both run the same kernels on
the same values.  Cases: fused rms + RoPE self-attention, cross-attention with
rms, GQA and key padding, no normalisation, the VAE's head_dim 384, and a
q-only normalisation whose q copy alone fits the array although q and k
together would not.  It also checks the size limit and the status query.
This file is collected last (tests/test_zz_*), and it sets up everything it
uses itself, so it passes alone in a fresh process or after the other tests.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIMIT = 32 << 20  # bytes of the fixed array


def _desc_for(ex, q, k, v, out, **kw):
    b, sq, h, d = q.shape
    desc = ex.make_desc(heads=h, query_count=sq, key_count=k.shape[1], head_dim=d,
                        key_value_heads=k.shape[2], batch=b, **kw)
    for name, t in (("q", q), ("k", k), ("v", v), ("o", out)):
        sb, st, sh, _ = t.stride()
        setattr(desc, f"{name}_batch_stride", sb)
        setattr(desc, f"{name}_tok_stride", st)
        setattr(desc, f"{name}_head_stride", sh)
    return desc


def test_noalloc_is_bit_identical_to_the_allocating_entry_point():
    import torch

    import animaxs_b200 as ax
    from animaxs_b200 import _lib

    lib = _lib.lib()
    torch.cuda.set_device(0)
    ex = ax.AttentionExecutor(0)
    stream = torch.cuda.current_stream()
    sh = ctypes.c_void_p(stream.cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(7)

    cases = [
        # DiT-style self-attention with rms + RoPE (4096 tokens, 8 heads)
        dict(b=1, sq=4096, sk=4096, h=8, hkv=8, d=128, kw=dict(qk_norm="rms_rope")),
        # cross-attention with rms, key padding and GQA (a different shape)
        dict(b=2, sq=777, sk=333, h=4, hkv=2, d=128, kw=dict(qk_norm="rms", kv_valid_len=200)),
        # no normalisation: the array is not used at all
        dict(b=1, sq=300, sk=1000, h=16, hkv=16, d=128, kw=dict(causal=False)),
        # the VAE's middle attention: one head of 384
        dict(b=1, sq=4096, sk=4096, h=1, hkv=1, d=384, kw=dict()),
        # q-only normalisation (k cached by the caller): 16384 x 16 x 128 fp16 of q
        # would not fit, 4096 x 16 x 128 does, and alone it fits although q + k would not
        dict(b=1, sq=4096, sk=8192, h=16, hkv=16, d=128, kw=dict(qk_norm="rms", qk_norm_targets="q")),
        # the first case again after all others: stale contents would show
        dict(b=1, sq=4096, sk=4096, h=8, hkv=8, d=128, kw=dict(qk_norm="rms_rope")),
    ]
    for i, c in enumerate(cases):
        q = torch.randn(c["b"], c["sq"], c["h"], c["d"], generator=g, device="cuda").half()
        k = torch.randn(c["b"], c["sk"], c["hkv"], c["d"], generator=g, device="cuda").half()
        v = torch.randn(c["b"], c["sk"], c["hkv"], c["d"], generator=g, device="cuda").half()
        kw = dict(c["kw"])
        if kw.get("qk_norm") == "rms_rope":
            kw["rope_table"] = torch.from_numpy(ax.qwen_rope(c["sk"])).cuda()
        desc = _desc_for(ex, q, k, v, q, **kw)
        need = ctypes.c_int64()
        assert lib.animaxs_attn_scratch_bytes(ctypes.byref(desc), ctypes.byref(need)) == 0
        assert need.value <= LIMIT, (i, need.value)
        ref = ex.attention(q, k, v, **kw)
        out = torch.full_like(q, float("nan"))
        desc = _desc_for(ex, q, k, v, out, **kw)
        rc = lib.animaxs_attn_forward_noalloc(ctypes.byref(desc), q.data_ptr(), k.data_ptr(),
                                              v.data_ptr(), out.data_ptr(), sh)
        assert rc == 0, f"case {i}: noalloc call failed with status {rc}"
        torch.cuda.synchronize()
        a = out.cpu().numpy().view(np.uint16)
        r = ref.cpu().numpy().view(np.uint16)
        assert np.isfinite(out.float().cpu().numpy()).all(), f"case {i}: non-finite output"
        assert np.array_equal(a, r), f"case {i}: {np.count_nonzero(a != r)} outputs differ from animaxs_attn_forward"
    assert lib.animaxs_attn_noalloc_status() == 0

    # beyond the fixed 32 MiB: rejected before any launch
    big_q = torch.empty(1, 16384, 16, 128, dtype=torch.float16, device="cuda")
    rope = torch.from_numpy(ax.qwen_rope(16384)).cuda()
    desc = _desc_for(ex, big_q, big_q, big_q, big_q, qk_norm="rms_rope", rope_table=rope)
    rc = lib.animaxs_attn_forward_noalloc(ctypes.byref(desc), big_q.data_ptr(), big_q.data_ptr(),
                                          big_q.data_ptr(), big_q.data_ptr(), sh)
    assert rc == _lib.ERR_SCRATCH_LIMIT == -9
    torch.cuda.synchronize()
    ex.close()
