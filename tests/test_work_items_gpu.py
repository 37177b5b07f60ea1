"""GPU: work items of the flash kernels.  A launch whose query-tile pairs would
leave more than half of the SMs idle deals single 128-row tiles instead (twice
the CTAs) and runs attn_s3_sm100.cu (one tile per CTA, three score buffers).
Every row's arithmetic is the same in all of them, so the output must be
BIT-IDENTICAL to the paired form.  The same inputs are run alone (single
tiles: few pairs) and as image 0 of a batch large enough to be dealt in pairs,
and compared; the single-tile launch is also checked against the oracle."""
import numpy as np
import pytest

from oracle import attn_oracle as ora
from tests.gpu_util import assert_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ex():
    from animaxs_b200 import AttentionExecutor
    e = AttentionExecutor(0)
    yield e
    e.close()


CASES = [
    # (name, q_len, kv_len, heads, kv_heads, head_dim, kw)
    ("dit_self_1024_rms_rope", 1024, 1024, 16, 16, 128, dict(qk_norm="rms_rope")),
    ("qwen_causal_gqa_padded", 512, 512, 16, 8, 128, dict(causal=True, qk_norm="rms_rope", kv_valid_len=300)),
    ("ragged_777x333", 777, 333, 8, 8, 128, dict(qk_norm="rms")),
    ("adapter_head_dim_64", 512, 512, 16, 16, 64, dict(qk_norm="rms_rope")),
]


@pytest.mark.parametrize("name,sq,sk,h,hkv,d,kw", CASES, ids=[c[0] for c in CASES])
def test_single_tile_items_equal_paired_items(ex, name, sq, sk, h, hkv, d, kw):
    import torch
    g = torch.Generator(device="cuda").manual_seed(17)
    q = torch.randn(1, sq, h, d, generator=g, device="cuda").half()
    k = torch.randn(1, sk, hkv, d, generator=g, device="cuda").half()
    v = torch.randn(1, sk, hkv, d, generator=g, device="cuda").half()
    kw = dict(kw)
    rope_np = None
    if kw.get("qk_norm") == "rms_rope":
        rope_np = ora.rope1d_table(max(sq, sk), 1.0e6, head_dim=d)
        kw["rope_table"] = torch.from_numpy(rope_np).cuda()
    pairs = (sq + 255) // 256
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert 2 * pairs * h <= sms, "the lone call must be dealt as single tiles"
    batch = (sms // (pairs * h)) + 1           # enough images for pairs
    assert 2 * pairs * h * batch > sms
    alone = ex.attention(q, k, v, **kw)
    big = [x.expand(batch, *x.shape[1:]).contiguous() for x in (q, k, v)]
    paired = ex.attention(*big, **kw)
    torch.cuda.synchronize()
    ex.synchronize()
    a = alone.cpu().numpy().view(np.uint16)
    b = paired[:1].cpu().numpy().view(np.uint16)
    assert np.array_equal(a, b), f"{name}: {np.count_nonzero(a != b)} outputs differ"
    want = ora.forward(*(x.cpu().numpy() for x in (q, k, v)), qk_norm=kw.get("qk_norm", "none"),
                       rope_table=rope_np, causal=kw.get("causal", False),
                       kv_valid_len=[kw["kv_valid_len"]] if "kv_valid_len" in kw else None)
    assert_parity(alone.float().cpu().numpy(), want, what=name)
