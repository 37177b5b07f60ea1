"""GPU: the cross-attention K/V cache (CrossKVCache, DiTBlockExecutor.swift:19-43,
reused across the 8 Euler steps at :1105-1161), through the C ABI.

The reference's contract is that a cache hit gives attention "byte-identical
inputs by construction" (:1114-1116).  Here: 8 cached steps equal 8 uncached
fused calls (q and k normalised in the prologue every step) BIT FOR BIT, for
several blocks, a batch of 2, a non-unit norm weight and the real context's
key padding; the projection fill is checked against the oracle's fp16
projection + RMSNorm."""
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


def _rand(g, *shape, scale=1.0):
    import torch
    return (scale * torch.randn(*shape, generator=g, device="cuda")).half()


@pytest.mark.parametrize("valid", [None, 47])
def test_eight_cached_steps_equal_uncached_bit_for_bit(ex, valid):
    import torch

    from animaxs_b200 import CrossKVCache
    g = torch.Generator(device="cuda").manual_seed(21)
    blocks, batch, ctx_tokens, heads = 3, 2, 512, 16
    k_raw = [_rand(g, batch, ctx_tokens, heads, 128) for _ in range(blocks)]
    v_raw = [_rand(g, batch, ctx_tokens, heads, 128) for _ in range(blocks)]
    qw = (1 + 0.2 * torch.randn(128, generator=g, device="cuda")).half()
    kw = (1 + 0.2 * torch.randn(128, generator=g, device="cuda")).half()
    cache = CrossKVCache(ex, blocks=blocks, batch=batch, tokens=ctx_tokens, kv_heads=heads)
    try:
        assert not any(cache.is_ready(b) for b in range(blocks))
        hits = 0
        for step in range(8):
            for b in range(blocks):
                q = _rand(g, batch, 1024, heads, 128)
                ref = ex.attention(q, k_raw[b], v_raw[b], qk_norm="rms", q_norm_weight=qw,
                                   k_norm_weight=kw, kv_valid_len=valid)
                if cache.is_ready(b):
                    hits += 1
                else:
                    cache.fill(b, k_raw[b], v_raw[b], k_norm_weight=kw)
                got = ex.attention(q, cache.k(b), cache.v(b), qk_norm="rms", qk_norm_targets="q",
                                   q_norm_weight=qw, kv_valid_len=valid)
                torch.cuda.synchronize()
                ex.synchronize()
                a, r = got.cpu().numpy().view(np.uint16), ref.cpu().numpy().view(np.uint16)
                assert np.array_equal(a, r), f"step {step} block {b}: {np.count_nonzero(a != r)} outputs differ"
        assert hits == 7 * blocks
        cache.reset()
        assert not cache.is_ready(0)
    finally:
        cache.close()


def test_fill_without_norm_copies_exactly(ex):
    import torch

    from animaxs_b200 import AttentionValidationError, CrossKVCache
    g = torch.Generator(device="cuda").manual_seed(3)
    cache = CrossKVCache(ex, blocks=2, batch=1, tokens=300, kv_heads=8, head_dim=64)
    try:
        big = _rand(g, 1, 300, 576)            # token stride 576: a strided source
        k, v = big[:, :, :512].unflatten(2, (8, 64)), _rand(g, 1, 300, 8, 64)
        cache.fill(1, k, v, k_norm=False)
        torch.cuda.synchronize()
        assert torch.equal(cache.k(1), k) and torch.equal(cache.v(1), v)
        assert cache.is_ready(1) and not cache.is_ready(0)
        cache.mark_ready(1, False)
        assert not cache.is_ready(1)
        with pytest.raises(AttentionValidationError):
            cache.fill(2, k, v)
    finally:
        cache.close()


def test_project_fills_normalised_k_and_v(ex):
    """The miss path from the adapter context: one fused GEMM, K RMS-normalised."""
    import torch

    from animaxs_b200 import CrossKVCache
    g = torch.Generator(device="cuda").manual_seed(9)
    tokens, ctx_dim, heads = 512, 1024, 16
    x = _rand(g, tokens, ctx_dim)
    w = _rand(g, 2 * heads * 128, ctx_dim, scale=ctx_dim ** -0.5)
    kw = (1 + 0.2 * torch.randn(128, generator=g, device="cuda")).half()
    cache = CrossKVCache(ex, blocks=1, batch=1, tokens=tokens, kv_heads=heads)
    try:
        cache.project(0, x, w, k_norm_weight=kw)
        torch.cuda.synchronize()
        ex.synchronize()
        assert cache.is_ready(0)
        want = ora.to_fp16_storage(ora.qkv_norm_projection(
            x.cpu().numpy(), w.cpu().numpy(), q_cols=0, k_cols=heads * 128, qk_norm="rms",
            k_norm_weight=kw.cpu().numpy(), tokens=tokens))
        got = np.concatenate([cache.k(0).reshape(tokens, -1).float().cpu().numpy(),
                              cache.v(0).reshape(tokens, -1).float().cpu().numpy()], axis=1)
        err = np.abs(got - want)
        assert (err <= 2e-3 + 2e-3 * np.abs(want)).all(), f"worst {err.max():.3e}"
        # cross-attention from the cached block against the fp32 oracle
        q = _rand(g, 1, 1024, heads, 128)
        out = ex.attention(q, cache.k(0), cache.v(0), qk_norm="rms", qk_norm_targets="q")
        torch.cuda.synchronize()
        kk = cache.k(0).float().cpu().numpy()
        vv = cache.v(0).float().cpu().numpy()
        qn = ora.rms_norm_heads(q.float().cpu().numpy())
        assert_parity(out.float().cpu().numpy(), ora.attention(qn, kk, vv), what="attention on projected cache")
    finally:
        cache.close()
