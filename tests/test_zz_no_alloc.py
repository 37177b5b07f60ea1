"""GPU test of animaxs_attn_forward_noalloc, the allocation-free entry point.

Who needs it: callers that must not have device memory allocated for them --
an application that reserves the GPU's memory up front and treats any later
cudaMalloc as a failure, a host runtime whose own allocator must own every
device allocation, or a latency-critical loop where an allocation (which can
synchronise the device) is unacceptable.  The entry point keeps the fused
prologue's normalised q/k in a fixed 32 MiB device array instead.

The test calls it through the C ABI twice in a row (different shapes and
values, so stale contents of the shared array would show) and compares each
output with the allocating entry point animaxs_attn_forward on the same
inputs, within the suite's tolerance.  It also checks the size limit.
This file is collected last (tests/test_zz_*), and it sets up everything it
uses itself, so it passes alone in a fresh process or after the other tests.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3


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


def test_noalloc_matches_allocating_entry_point_twice():
    import torch

    import animaxs_b200 as ax
    from animaxs_b200 import _lib

    lib = _lib.lib()
    torch.cuda.set_device(0)
    ex = ax.AttentionExecutor(0)
    stream = torch.cuda.current_stream()
    sh = ctypes.c_void_p(stream.cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(7)

    # call 1: DiT-style self-attention with rms + RoPE (4096 tokens, 8 heads)
    # call 2: cross-attention with rms, key padding and GQA (different shape)
    cases = [
        dict(b=1, sq=4096, sk=4096, h=8, hkv=8, kw=dict(qk_norm="rms_rope")),
        dict(b=2, sq=777, sk=333, h=4, hkv=2, kw=dict(qk_norm="rms", kv_valid_len=200)),
    ]
    for c in cases:
        q = torch.randn(c["b"], c["sq"], c["h"], 128, generator=g, device="cuda").half()
        k = torch.randn(c["b"], c["sk"], c["hkv"], 128, generator=g, device="cuda").half()
        v = torch.randn(c["b"], c["sk"], c["hkv"], 128, generator=g, device="cuda").half()
        kw = dict(c["kw"])
        if kw.get("qk_norm") == "rms_rope":
            kw["rope_table"] = torch.from_numpy(ax.qwen_rope(c["sk"])).cuda()
        ref = ex.attention(q, k, v, **kw)
        out = torch.full_like(q, float("nan"))
        desc = _desc_for(ex, q, k, v, out, **kw)
        rc = lib.animaxs_attn_forward_noalloc(ctypes.byref(desc), q.data_ptr(), k.data_ptr(),
                                              v.data_ptr(), out.data_ptr(), sh)
        assert rc == 0, f"noalloc call failed with status {rc}"
        torch.cuda.synchronize()
        diff = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert float(diff.max()) <= MAX_ABS, f"max-abs {float(diff.max()):.3e}"

    # beyond the fixed 32 MiB: rejected before any launch
    big_q = torch.empty(1, 16384, 16, 128, dtype=torch.float16, device="cuda")
    rope = torch.from_numpy(ax.qwen_rope(16384)).cuda()
    desc = _desc_for(ex, big_q, big_q, big_q, big_q, qk_norm="rms_rope", rope_table=rope)
    rc = lib.animaxs_attn_forward_noalloc(ctypes.byref(desc), big_q.data_ptr(), big_q.data_ptr(),
                                          big_q.data_ptr(), big_q.data_ptr(), sh)
    assert rc == _lib.ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    ex.close()
    np.testing.assert_equal(rc, -9)
