"""GPU: the q/k normalisation prologue (qk_norm.cu) gives a row the same bits
whatever else shares its CTA.

A CTA normalises one token's rows, dealt to row slots of 8 lanes; each warp's
4 slots share the token's rotation blocks (a quarter loaded by each, the rest
by shuffle) and the weights are loaded once per thread.  A row's arithmetic
(fp32 statistics, the shared weight, the split-half rotation of
AnimaKernels.metal:660-729) must not depend on how many heads the call has,
on the row stride, or on which slot the row lands in.  Here 40 heads of a
token (8 slots in two warps, two rounds of rows) are compared with the first
16 of the same heads run alone (4 slots in one warp, strided rows), BIT FOR BIT,
for RMSNorm and RMSNorm + RoPE at head_dim 128 and 64, and both against the
oracle."""
import numpy as np
import pytest

from oracle import attn_oracle as ora

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ex():
    from animaxs_b200 import AttentionExecutor
    e = AttentionExecutor(0)
    yield e
    e.close()


@pytest.mark.parametrize("head_dim", [128, 64])
@pytest.mark.parametrize("rope", [False, True], ids=["rms", "rms_rope"])
def test_row_bits_do_not_depend_on_the_call_shape(ex, head_dim, rope):
    import torch
    tokens, wide, narrow = 300, 40, 16
    g = torch.Generator(device="cuda").manual_seed(head_dim + int(rope))
    x = (torch.randn(tokens, wide, head_dim, generator=g, device="cuda") * 3).half()
    w = torch.linspace(0.5, 1.5, head_dim, device="cuda").half()
    table_np = ora.rope1d_table(tokens, 1.0e6, head_dim=head_dim)
    table = torch.from_numpy(table_np).cuda()
    stream = torch.cuda.current_stream()
    out_wide = torch.full_like(x, float("nan"))
    out_narrow = torch.full_like(x, float("nan"))
    stride = wide * head_dim
    if rope:
        ex.rms_rope_split_half(stream, x, out_wide, w, table, tokens=tokens, heads=wide, head_dim=head_dim)
        ex.rms_rope_split_half(stream, x, out_narrow, w, table, tokens=tokens, heads=narrow,
                               head_dim=head_dim, row_stride=stride)
    else:
        ex.rmsnorm_heads_half(stream, x, out_wide, w, tokens=tokens, heads=wide, head_dim=head_dim)
        ex.rmsnorm_heads_half(stream, x, out_narrow, w, tokens=tokens, heads=narrow, head_dim=head_dim,
                              row_stride=stride)
    torch.cuda.synchronize()
    a = out_wide[:, :narrow].cpu().numpy().view(np.uint16)
    b = out_narrow[:, :narrow].cpu().numpy().view(np.uint16)
    assert np.array_equal(a, b), f"{np.count_nonzero(a != b)} of {a.size} values differ"
    # the heads past the 16 were not written by the narrow call
    assert torch.isnan(out_narrow[:, narrow:]).all()
    ref = ora.rms_norm_heads(x.float().cpu().numpy()[None], w.float().cpu().numpy())
    if rope:
        ref = ora.apply_split_half_rope(ref, table_np)
    np.testing.assert_allclose(out_wide.float().cpu().numpy(), ora.to_fp16_storage(ref[0]), atol=4e-3, rtol=2e-3)
