"""GPU parity of the wide-head attention kernel (head_dim 384 and 256,
attn_wide_sm100.cu) against the CPU oracle, through the C ABI.

The reference's wide caller is the VAE decoder's middle attention
(VAEDecoder.swift:351-410 -> AttentionExecutor.execute, head-major layout).
The launch splits a query tile's keys over a cluster of 1, 2 or 4 CTAs
depending on how many query tiles there are; the shapes below reach all
three, including splits left without key tiles (causal, early query tiles)."""
import numpy as np
import pytest

from oracle import attn_oracle as ora
from oracle import inputs
from tests.gpu_util import assert_parity, run_case, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ex():
    from animaxs_b200 import AttentionExecutor
    e = AttentionExecutor(0)
    yield e
    e.close()


def test_vae_middle_attention_reference_call(ex):
    """The reference's own call: Q/K/V are contiguous [positions, 384] blocks
    of one split buffer, passed with byte offsets, heads 1, head-major."""
    import torch
    case = inputs.vae_attention(seed=11)
    pos, ch = 64 * 64, 384
    split = torch.cat([to_dev(case.q[0, :, 0]), to_dev(case.k[0, :, 0]), to_dev(case.v[0, :, 0])])
    out = torch.full((pos, ch), float("nan"), dtype=torch.float16, device="cuda")
    half = 2
    ex.execute(split, split, split, out, heads=1, query_count=pos, key_count=pos, head_dim=ch,
               key_offset=pos * ch * half, value_offset=pos * ch * 2 * half, causal=False)
    got = out.float().cpu().numpy()[None, :, None, :]
    assert_parity(got, case.oracle(), what="VAE middle attention 64x64 x 384")


@pytest.mark.parametrize(
    "d,b,h,hkv,sq,sk,causal,layout",
    [
        (384, 1, 1, 1, 1, 1, False, "token"),       # one row, one key
        (384, 1, 1, 1, 129, 300, False, "token"),   # ragged, 3 key tiles: no split
        (384, 1, 1, 1, 2048, 2048, True, "head"),   # 4-way split, empty splits early
        (384, 1, 2, 2, 1000, 1000, True, "token"),  # causal, ragged tail
        (384, 2, 1, 1, 1024, 4096, False, "head"),  # cross-shaped, 4-way split
        (256, 1, 4, 2, 1280, 1280, False, "token"), # GQA, 2-way split
        (256, 3, 2, 2, 640, 777, False, "head"),    # batched, ragged keys
        (256, 8, 8, 8, 512, 512, False, "token"),   # 256 query tiles: no split, several waves
    ])
def test_wide_shapes(ex, d, b, h, hkv, sq, sk, causal, layout):
    q, k, v = inputs.draw_qkv(d + sq + 7 * sk + b, (b, sq, h, d), (b, sk, hkv, d))
    case = inputs.Case(f"wide{d}", q, k, v, causal=causal)
    out = run_case(ex, case, layout=layout)
    assert_parity(out, case.oracle(), what=f"d={d} B={b} H={h}/{hkv} {sq}x{sk} causal={causal}")


def test_wide_key_padding(ex):
    """kv_valid_len (scalar) and kv_valid_lens (per batch, device) at head_dim 384."""
    import torch
    q, k, v = inputs.draw_qkv(3, (3, 700, 1, 384), (3, 1500, 1, 384))
    case = inputs.Case("wide_pad", q, k, v, kv_valid_len=[1111] * 3)
    assert_parity(run_case(ex, case), case.oracle(), what="scalar kv_valid_len 1111 of 1500")
    lens = [1500, 1, 640]
    case = inputs.Case("wide_pad_b", q, k, v, kv_valid_len=lens)
    dl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = ex.attention(to_dev(q), to_dev(k), to_dev(v), kv_valid_lens=dl)
    torch.cuda.synchronize()
    assert_parity(out.float().cpu().numpy(), case.oracle(), what="per-batch valid lengths")


def test_wide_split_matches_unsplit(ex):
    """The same query rows computed with the keys split over a cluster (one
    head) and without (enough heads that the launch does not split) agree to
    the fp16 output rounding."""
    import torch
    q, k, v = inputs.draw_qkv(21, (1, 2048, 1, 384), (1, 2048, 1, 384))
    qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)
    split = ex.attention(qd, kd, vd)
    many = ex.attention(qd.expand(1, 2048, 40, 384).contiguous(), kd, vd)
    torch.cuda.synchronize()
    diff = (split.float() - many[:, :, 7:8].float()).abs().max().item()
    assert diff <= 2e-3, diff
    assert_parity(split.float().cpu().numpy(), ora.attention(q, k, v), what="split vs oracle")


def test_wide_rejects_fused_norm(ex):
    import torch
    from animaxs_b200 import AttentionValidationError
    x = torch.zeros(1, 128, 1, 384, dtype=torch.float16, device="cuda")
    with pytest.raises(AttentionValidationError, match="headDim 128 or 64"):
        ex.attention(x, x, x, qk_norm="rms")


def test_wide_output_sentinels_untouched(ex):
    """Rows past q_len and columns outside the head are never written."""
    import torch
    q, k, v = inputs.draw_qkv(4, (1, 200, 1, 384), (1, 600, 1, 384))
    out_full = torch.full((1, 256, 1, 400), 7.0, dtype=torch.float16, device="cuda")
    out = out_full[:, :200, :, :384]
    ex.attention(to_dev(q), to_dev(k), to_dev(v), out)
    torch.cuda.synchronize()
    assert torch.all(out_full[:, 200:] == 7.0)
    assert torch.all(out_full[..., 384:] == 7.0)
    assert_parity(out.float().cpu().numpy(), ora.attention(q, k, v), what="strided output")
