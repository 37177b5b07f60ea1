"""Seeded synthetic inputs for the five benchmark configurations.

TEST INFRASTRUCTURE ONLY (used by ``tests/``, ``smoke()`` and the CPU legs of
``bench.py``).  Inputs are drawn on the CPU with ``torch.Generator`` so that
this container, the GPU box and the golden-fixture script all see identical
values: ``g = torch.Generator().manual_seed(seed)``; ``q, k, v = randn(...)``
in that order as fp32, then rounded to fp16.  Shapes are token-major
``[B, S, H, D]`` (D = 128; 64 for the LLM adapter; 384 for the VAE) -- the layout the
reference's projections produce
(``DiTBlockExecutor.swift:1097-1131``, ``QwenEncoderMetal.swift:245-262``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import attn_oracle as ora


@dataclass
class Case:
    name: str
    q: np.ndarray            # fp16 [B, Sq, Hq, D]
    k: np.ndarray            # fp16 [B, Sk, Hkv, D]
    v: np.ndarray            # fp16 [B, Sk, Hkv, D]
    qk_norm: str = "none"
    rope_table: np.ndarray | None = None
    causal: bool = False
    kv_valid_len: list | None = None
    meta: dict = field(default_factory=dict)

    @property
    def heads(self):
        return self.q.shape[2]

    @property
    def kv_heads(self):
        return self.k.shape[2]

    def oracle(self, rows=None):
        return ora.forward(self.q, self.k, self.v, qk_norm=self.qk_norm,
                           rope_table=self.rope_table, causal=self.causal,
                           kv_valid_len=self.kv_valid_len, rows=rows)

    def flops(self) -> float:
        """Algorithmic FLOPs: 4 * (valid q-k pairs) * D * Hq."""
        b, sq, hq, d = self.q.shape
        sk = self.k.shape[1]
        total = 0
        valid = self.kv_valid_len or [sk] * b
        for vb in valid:
            vb = min(int(vb), sk)
            if self.causal:
                rows = np.arange(sq)
                total += int(np.minimum(rows + 1, vb).sum())
            else:
                total += sq * vb
        return 4.0 * total * d * hq


def draw_qkv(seed: int, q_shape, kv_shape):
    import torch
    g = torch.Generator().manual_seed(int(seed))
    q = torch.randn(q_shape, generator=g, dtype=torch.float32).half().numpy()
    k = torch.randn(kv_shape, generator=g, dtype=torch.float32).half().numpy()
    v = torch.randn(kv_shape, generator=g, dtype=torch.float32).half().numpy()
    return q, k, v


def dit_self(seed: int = 0, grid=(1, 32, 32), heads: int = 16, batch: int = 1) -> Case:
    """Configs 1/5 (and the self half of config 4): rms + 3-D RoPE, non-causal."""
    t, h, w = grid
    s = t * h * w
    q, k, v = draw_qkv(seed, (batch, s, heads, ora.HEAD_DIM), (batch, s, heads, ora.HEAD_DIM))
    return Case(f"dit_self_{s}", q, k, v, qk_norm="rms_rope",
                rope_table=ora.dit_rope_table(t, h, w), meta={"grid": grid, "seed": seed})


def dit_cross(seed: int = 0, q_len: int = 4096, kv_len: int = 512, heads: int = 16,
              kv_valid: int | None = 128, batch: int = 1) -> Case:
    """Config 2: rms only; ``kv_valid`` keys kept (None = unmasked reference semantics)."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    q = torch.randn((batch, q_len, heads, ora.HEAD_DIM), generator=g).half().numpy()
    k = torch.randn((batch, kv_len, heads, ora.HEAD_DIM), generator=g).half().numpy()
    v = torch.randn((batch, kv_len, heads, ora.HEAD_DIM), generator=g).half().numpy()
    valid = None if kv_valid is None else [kv_valid] * batch
    return Case(f"dit_cross_{q_len}x{kv_len}", q, k, v, qk_norm="rms",
                kv_valid_len=valid, meta={"seed": seed})


def qwen_prefill(layer: int = 0, seq_len: int = 512, heads: int = 16, kv_heads: int = 8,
                 valid: int | None = 300) -> Case:
    """Config 3: seed 1 + layer; rms + 1-D RoPE (theta 1e6); causal + right padding."""
    q, k, v = draw_qkv(1 + layer, (1, seq_len, heads, ora.HEAD_DIM),
                       (1, seq_len, kv_heads, ora.HEAD_DIM))
    return Case(f"qwen_l{layer}", q, k, v, qk_norm="rms_rope",
                rope_table=ora.rope1d_table(seq_len, 1.0e6), causal=True,
                kv_valid_len=None if valid is None else [valid], meta={"layer": layer})


def adapter_attention(seed: int = 0, target_tokens: int = 512, context_tokens: int | None = None,
                      heads: int = 16, batch: int = 1) -> Case:
    """LLM adapter attention (LLMAdapterMetal.swift:361-404): 16 heads of 64,
    q and k through rms_rope_adapter64 (RMSNorm, unit weights here, then the
    adapter's RoPE), non-causal.  Self-attention over the target tokens, or
    cross-attention from them to ``context_tokens`` rows (the Qwen context);
    both at most 512 tokens (LLMAdapterMetal.swift:7,45-46)."""
    kv = target_tokens if context_tokens is None else context_tokens
    q, k, v = draw_qkv(seed, (batch, target_tokens, heads, ora.ADAPTER_HEAD_DIM),
                       (batch, kv, heads, ora.ADAPTER_HEAD_DIM))
    name = f"adapter_{target_tokens}x{kv}"
    return Case(name, q, k, v, qk_norm="rms_rope",
                rope_table=ora.adapter_rope_table(max(target_tokens, kv)))


def vae_attention(seed: int = 0, latent: int = 64, channels: int = 384, batch: int = 1) -> Case:
    """The VAE decoder's middle attention (VAEDecoder.swift:351-410): one head
    of ``channels`` over the ``latent x latent`` positions, non-causal, no q/k
    norm, scale 1/sqrt(channels).  Q/K/V stand in for the normalised 1x1 to_qkv
    projection of a latent (unit-variance per channel)."""
    s = latent * latent
    q, k, v = draw_qkv(seed, (batch, s, 1, channels), (batch, s, 1, channels))
    return Case(f"vae_attn_{latent}x{latent}", q, k, v, meta={"seed": seed, "latent": latent})


def workload_seed(prompt: int, step: int, block: int) -> int:
    """Config 4 seeding: prompt p's (step, block) inputs use seed p + 8*(28*step + block).

    Step 0 / block 0 of prompt p is drawn from seed p, as the configuration
    states; every other block gets its own seed so that any (step, block)
    can be regenerated without replaying the whole trajectory.
    """
    return int(prompt) + 8 * (28 * int(step) + int(block))


def workload_block(prompt: int, step: int, block: int):
    """Config 4 block inputs: self (rms+rope3d 64x64) then cross (rms, unmasked)."""
    import torch
    g = torch.Generator().manual_seed(workload_seed(prompt, step, block))
    shp = (1, 4096, 16, ora.HEAD_DIM)
    cshp = (1, 512, 16, ora.HEAD_DIM)
    sq = torch.randn(shp, generator=g).half().numpy()
    sk = torch.randn(shp, generator=g).half().numpy()
    sv = torch.randn(shp, generator=g).half().numpy()
    cq = torch.randn(shp, generator=g).half().numpy()
    ck = torch.randn(cshp, generator=g).half().numpy()
    cv = torch.randn(cshp, generator=g).half().numpy()
    self_case = Case("wl_self", sq, sk, sv, qk_norm="rms_rope",
                     rope_table=ora.dit_rope_table(1, 64, 64))
    cross_case = Case("wl_cross", cq, ck, cv, qk_norm="rms")
    return self_case, cross_case


def proj_qkv(seed: int, images: int = 2, tokens: int = 64, k: int = 256, q_heads: int = 2,
             k_heads: int = 2, v_cols: int = 256):
    """Inputs of the fused q|k|v projection: x [images*tokens, k] ~ N(0, 1),
    w [q_heads*128 + k_heads*128 + v_cols, k] ~ N(0, 1/k) (unit-variance
    projections), norm weights ~ 1 + N(0, 0.1^2); fp16.  Drawn in that order."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    n = (q_heads + k_heads) * 128 + v_cols
    x = torch.randn(images * tokens, k, generator=g).half().numpy()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).half().numpy()
    qw = (1 + 0.1 * torch.randn(128, generator=g)).half().numpy()
    kw = (1 + 0.1 * torch.randn(128, generator=g)).half().numpy()
    return x, w, qw, kw


def proj_gate(seed: int, images: int = 2, tokens: int = 64, k: int = 256, n: int = 256):
    """Inputs of the out-projection + gated residual: x [images*tokens, k] fp16,
    w [n, k] ~ N(0, 1/k) fp16, residual [images*tokens, n] fp32, gate
    [images, n] fp32 ~ N(0, 0.5^2).  Drawn in that order."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    x = torch.randn(images * tokens, k, generator=g).half().numpy()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).half().numpy()
    residual = torch.randn(images * tokens, n, generator=g).numpy()
    gate = (0.5 * torch.randn(images, n, generator=g)).numpy()
    return x, w, residual, gate


def quant_weight(seed: int, rows: int, k: int, bits: int, packed_stride: int | None = None):
    """Seeded W4 / W8 weight buffers in the reference's pack layout
    (scripts/pack_anima.py:217-296): codes ``[rows][packed_stride]`` uint8 (W4:
    two per byte, even column low), fp16 ``scale`` / ``zero`` ``[rows][ceil(k / 64)]``
    with the magnitudes a quantized DiT weight has (span / qmax, group minimum)."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    need = (k + 1) // 2 if bits == 4 else k
    stride = need if packed_stride is None else packed_stride
    packed = torch.randint(0, 256, (rows, stride), generator=g, dtype=torch.int32).to(torch.uint8).numpy()
    groups = (k + 63) // 64
    qmax = 15.0 if bits == 4 else 255.0
    span = torch.rand(rows, groups, generator=g) * 0.2 + 1e-3
    lo = -span * torch.rand(rows, groups, generator=g)
    scale = (span / qmax).to(torch.float16).numpy()
    zero = lo.to(torch.float16).numpy()
    return packed, scale, zero


def proj_x(seed: int, rows: int, k: int) -> np.ndarray:
    """Seeded fp16 activations ``[rows, k]`` for a projection."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    return torch.randn(rows, k, generator=g).half().numpy()
