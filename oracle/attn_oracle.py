"""CPU oracle for the AnimaXS attention hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against; it is imported by ``tests/``, by ``__graft_entry__.smoke()``
and by the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` and by
nothing else.  The product (``animaxs_b200`` + ``libanimaxs_attn.so``) never
calls it and has no CPU fallback.

It is a numpy restatement, in fp32, of the reference's own PyTorch CPU oracles
and Swift/Metal kernels for this path (citations are ``path:line`` inside the
AnimaXS project):

* per-head RMSNorm ........ ``scripts/dit_source_oracle.py:80-85`` (``rms_norm``),
                            ``scripts/qwen_comfy_oracle.py:138-140``,
                            ``AnimaXS/Shaders/AnimaKernels.metal:660-689``
* split-half RoPE ......... ``scripts/dit_source_oracle.py:174-194``,
                            ``AnimaXS/Shaders/AnimaKernels.metal:696-729``,
                            ``scripts/qwen_comfy_oracle.py:122-135`` (same rotation)
* 3-D RoPE table .......... ``scripts/dit_source_oracle.py:126-171`` (``dit_rope``),
                            ``AnimaXS/Runtime/Text/DitRoPE.swift:58-107``
* 1-D (Qwen) RoPE table ... ``scripts/qwen_comfy_oracle.py:95-119``,
                            ``AnimaXS/Runtime/Metal/QwenEncoderMetal.swift:126-142``
* GQA head map ............ ``AnimaXS/Runtime/Metal/AttentionExecutor.swift:222``,
                            ``scripts/qwen_comfy_oracle.py:87-92`` (repeat_interleave)
* attention ............... ``scripts/dit_source_oracle.py:108-120``
                            (``scaled_dot_product``: fp32 scores, fp32 softmax),
                            ``scripts/qwen_comfy_oracle.py:146-161`` (additive mask
                            path of ``attention_pytorch``)
* masks ................... ``scripts/qwen_comfy_oracle.py:238-248``: additive
                            ``finfo.min / 4`` for causal (``triu(1)``) and key padding
* score-health probe ...... ``AnimaXS/Shaders/AnimaKernels.metal:1738-1830``
                            (``attention_softmax_rows_probe``; slot layout
                            ``AnimaXS/Runtime/Diagnostics/NumericalMonitor.swift:136-161``)
* W4/W8 weight decode ..... ``scripts/animapk_cuda/quant.py:32-76``
                            (``decode_w4_matrix`` / ``decode_w8_matrix``),
                            ``AnimaXS/Shaders/AnimaKernels.metal:19-67``
                            (``dequant_w4_to_half`` / ``dequant_w8_to_half``)

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
functions (imported from the AnimaXS ``scripts/`` directory) on seeded inputs
and commits their outputs as fixtures; ``tests/test_oracle_golden.py`` checks
this module against them.

Everything is computed in float32 from fp16-rounded inputs, the way the
north-star tolerance (max-abs 2e-3, mean-abs 2e-4 after fp16 storage) is
defined.
"""

from __future__ import annotations

import numpy as np

HEAD_DIM = 128
ROPE_PAIRS = HEAD_DIM // 2
EPS = 1e-6
# scripts/qwen_comfy_oracle.py:241,245 -- additive mask value finfo(dtype).min / 4
MASK_VALUE = np.float32(np.finfo(np.float32).min / 4)

# DiT 3-D RoPE axis split (DitRoPE.swift:27-39, dit_source_oracle.py:130-132):
DIM_H = HEAD_DIM // 6 * 2          # 42 dims -> 21 pairs
DIM_W = DIM_H                      # 42 dims -> 21 pairs
DIM_T = HEAD_DIM - 2 * DIM_H       # 44 dims -> 22 pairs


# ---------------------------------------------------------------------------
# Normalisation and rotation
# ---------------------------------------------------------------------------
def rms_norm_heads(x: np.ndarray, weight: np.ndarray | None = None, eps: float = EPS) -> np.ndarray:
    """Per-(token, head) RMSNorm over the last axis with fp32 statistics.

    dit_source_oracle.py:80-85: ``xf * rsqrt(mean(xf^2) + eps) * weight``.
    The shared ``[head_dim]`` weight is broadcast over every head
    (AnimaKernels.metal:660-689, weight indexed by ``d`` only).
    """
    xf = np.asarray(x, dtype=np.float32)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    out = xf * (np.float32(1.0) / np.sqrt(var + np.float32(eps)))
    if weight is not None:
        out = out * np.asarray(weight, dtype=np.float32)
    return out.astype(np.float32)


def apply_split_half_rope(x: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Split-half rotation of pairs ``(p, p + D/2)`` with a ``[S, D/2, 2, 2]`` table.

    dit_source_oracle.py:174-194 and AnimaKernels.metal:718-728:
    ``out[p] = cos*a - sin*b``, ``out[p+64] = sin*a + cos*b`` with
    ``a = x[p]``, ``b = x[p+64]``, ``cos = table[t,p,0,0]``, ``sin = table[t,p,1,0]``.

    ``x`` is ``[B, S, H, D]`` (token-major); the table row is the token index.
    """
    xf = np.asarray(x, dtype=np.float32)
    half = xf.shape[-1] // 2
    s = xf.shape[1]
    cos = table[:s, :half, 0, 0][None, :, None, :]
    sin = table[:s, :half, 1, 0][None, :, None, :]
    a = xf[..., :half]
    b = xf[..., half:]
    out = np.empty_like(xf)
    out[..., :half] = cos * a - sin * b
    out[..., half:] = sin * a + cos * b
    return out


# ---------------------------------------------------------------------------
# RoPE tables ([tokens, 64, 2, 2] fp32, each block [cos, -sin, sin, cos])
# ---------------------------------------------------------------------------
def _blocks(angle: np.ndarray) -> np.ndarray:
    c = np.cos(angle).astype(np.float32)
    s = np.sin(angle).astype(np.float32)
    return np.stack([c, -s, s, c], axis=-1)


def dit_rope_table(T: int = 1, H: int = 32, W: int = 32) -> np.ndarray:
    """3-D RoPE table, dit_source_oracle.py:126-171 / DitRoPE.swift:58-107.

    t/h/w = 44/42/42 dims (22/21/21 pairs) in that order; theta_hw =
    10000 * 4^(42/40) narrowed to fp32, theta_t = 10000; token index
    ``(t*H + h)*W + w``.
    """
    h_theta = np.float32(10000.0 * 4.0 ** (DIM_H / (DIM_H - 2)))
    w_theta = np.float32(10000.0 * 4.0 ** (DIM_W / (DIM_W - 2)))
    t_theta = np.float32(10000.0 * 1.0 ** (DIM_T / (DIM_T - 2)))
    rng_h = np.arange(0, DIM_H, 2)[: DIM_H // 2].astype(np.float32) / np.float32(DIM_H)
    rng_w = np.arange(0, DIM_W, 2)[: DIM_W // 2].astype(np.float32) / np.float32(DIM_W)
    rng_t = np.arange(0, DIM_T, 2)[: DIM_T // 2].astype(np.float32) / np.float32(DIM_T)
    f_h = (np.float32(1.0) / np.power(h_theta, rng_h)).astype(np.float32)
    f_w = (np.float32(1.0) / np.power(w_theta, rng_w)).astype(np.float32)
    f_t = (np.float32(1.0) / np.power(t_theta, rng_t)).astype(np.float32)
    seq = np.arange(max(H, W, T), dtype=np.float32)
    e_t = _blocks(np.outer(seq[:T], f_t))  # [T, 22, 4]
    e_h = _blocks(np.outer(seq[:H], f_h))  # [H, 21, 4]
    e_w = _blocks(np.outer(seq[:W], f_w))  # [W, 21, 4]
    em = np.concatenate([
        np.broadcast_to(e_t[:, None, None], (T, H, W, DIM_T // 2, 4)),
        np.broadcast_to(e_h[None, :, None], (T, H, W, DIM_H // 2, 4)),
        np.broadcast_to(e_w[None, None, :], (T, H, W, DIM_W // 2, 4)),
    ], axis=-2)
    return np.ascontiguousarray(em.reshape(T * H * W, ROPE_PAIRS, 2, 2), dtype=np.float32)


def rope1d_table(seq_len: int, theta: float = 1.0e6, head_dim: int = HEAD_DIM) -> np.ndarray:
    """1-D NeoX RoPE table in the same block layout (Qwen3, theta 1e6).

    qwen_comfy_oracle.py:95-119 (``inv = 1/theta^(2p/D)``, angle = pos * inv)
    laid out as QwenEncoderMetal.swift:126-142 does.
    """
    num = np.arange(0, head_dim, 2).astype(np.float32)
    inv = (np.float32(1.0) / np.power(np.float32(theta), num / np.float32(head_dim))).astype(np.float32)
    pos = np.arange(seq_len, dtype=np.float32)
    return np.ascontiguousarray(_blocks(np.outer(pos, inv)).reshape(seq_len, head_dim // 2, 2, 2))


# LLM adapter attention heads are 64 wide (LLMAdapterMetal.swift:9-10).
ADAPTER_HEAD_DIM = 64


def adapter_rope_table(tokens: int) -> np.ndarray:
    """The LLM adapter's RoPE table, LLMAdapterMetal.swift:162-178 (makeRope).

    32 pairs per token: ``inverse = 1 / pow(10000, 2p / 64)`` and
    ``angle = token * inverse`` in fp32, blocks ``[cos, -sin, sin, cos]``;
    consumed by rms_rope_adapter64 (AnimaKernels.metal:733-763), which rotates
    the pairs ``(p, p + 32)`` exactly as ``apply_split_half_rope`` does for a
    64-wide head.  Same construction as the 1-D table with theta 1e4 and
    head_dim 64.
    """
    return rope1d_table(tokens, theta=1.0e4, head_dim=ADAPTER_HEAD_DIM)


# ---------------------------------------------------------------------------
# GQA and attention
# ---------------------------------------------------------------------------
def gqa_kv_head(query_head: int, query_heads: int, kv_heads: int) -> int:
    """AttentionExecutor.swift:222 -- ``kvHead = head / (heads / kvHeads)``."""
    if kv_heads <= 0 or query_heads % kv_heads:
        raise ValueError("query heads must be a positive multiple of kv heads")
    return query_head // (query_heads // kv_heads)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, *, scale: float | None = None,
              causal: bool = False, kv_valid_len=None, rows=None,
              q_block: int = 512) -> np.ndarray:
    """Scaled dot-product attention, fp32 scores and softmax.

    ``q``: ``[B, Sq, Hq, D]``; ``k``/``v``: ``[B, Sk, Hkv, D]``.  Returns
    ``[B, len(rows), Hq, D]`` fp32 (``rows`` defaults to every query row).

    Follows dit_source_oracle.py:108-120 (scores = q @ k^T * scale, fp32
    softmax, probs @ v) with the additive ``finfo.min/4`` masks of
    qwen_comfy_oracle.py:238-248 (causal ``j > i`` and key padding
    ``j >= kv_valid_len[b]``).  Query rows are processed in blocks so the full
    score matrix is never materialised (the 16K-token case would need 17 GiB).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    bsz, sq, hq, d = q.shape
    sk, hkv = k.shape[1], k.shape[2]
    if scale is None:
        scale = d ** -0.5
    scale = np.float32(scale)
    rows = np.arange(sq) if rows is None else np.asarray(rows)
    if kv_valid_len is None:
        valid = [sk] * bsz
    elif np.isscalar(kv_valid_len):
        valid = [int(kv_valid_len)] * bsz
    else:
        valid = [int(x) for x in kv_valid_len]
    out = np.zeros((bsz, len(rows), hq, d), dtype=np.float32)
    cols = np.arange(sk)
    for b in range(bsz):
        for h in range(hq):
            kvh = gqa_kv_head(h, hq, hkv)
            kt = np.ascontiguousarray(k[b, :, kvh, :].T)
            vh = np.ascontiguousarray(v[b, :, kvh, :])
            for r0 in range(0, len(rows), q_block):
                rr = rows[r0:r0 + q_block]
                s = (q[b, rr, h, :] @ kt) * scale
                masked = np.broadcast_to(cols[None, :] >= valid[b], s.shape)
                if causal:
                    masked = masked | (cols[None, :] > rr[:, None])
                s = np.where(masked, s + MASK_VALUE, s).astype(np.float32)
                m = s.max(axis=-1, keepdims=True)
                p = np.exp(s - m, dtype=np.float32)
                p /= p.sum(axis=-1, keepdims=True, dtype=np.float32)
                out[b, r0:r0 + len(rr), h, :] = p @ vh
    return out


def forward(q, k, v, *, qk_norm: str = "none", q_norm_weight=None, k_norm_weight=None,
            eps: float = EPS, rope_table=None, causal: bool = False, kv_valid_len=None,
            scale: float | None = None, rows=None) -> np.ndarray:
    """The fused operator the CUDA path implements, restated on the CPU.

    ``qk_norm`` is ``"none"``, ``"rms"`` (cross-attention q/k,
    DiTBlockExecutor.swift:1608-1626 -> AnimaKernels.metal:660-689) or
    ``"rms_rope"`` (DiT self q/k and Qwen q/k, AnimaKernels.metal:696-729).
    Inputs are ``[B, S, H, D]`` (token-major); output ``[B, len(rows), Hq, D]``.
    """
    qf = np.asarray(q, dtype=np.float32)
    kf = np.asarray(k, dtype=np.float32)
    if qk_norm in ("rms", "rms_rope"):
        qf = rms_norm_heads(qf, q_norm_weight, eps)
        kf = rms_norm_heads(kf, k_norm_weight, eps)
    if qk_norm == "rms_rope":
        if rope_table is None:
            raise ValueError("rms_rope needs a rope table")
        qf = apply_split_half_rope(qf, rope_table)
        kf = apply_split_half_rope(kf, rope_table)
    elif qk_norm not in ("none", "rms"):
        raise ValueError(f"unknown qk_norm {qk_norm!r}")
    return attention(qf, kf, v, scale=scale, causal=causal, kv_valid_len=kv_valid_len, rows=rows)


def to_fp16_storage(x: np.ndarray) -> np.ndarray:
    """Round an fp32 result the way an fp16 output buffer stores it."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def parity(actual_fp16: np.ndarray, oracle_fp32: np.ndarray) -> tuple[float, float]:
    """(max-abs, mean-abs) of an fp16 result against the fp16-stored oracle."""
    a = np.asarray(actual_fp16, dtype=np.float32)
    e = to_fp16_storage(oracle_fp32)
    diff = np.abs(a - e)
    return float(diff.max()), float(diff.mean())


# ---------------------------------------------------------------------------
# The projections on either side of attention (fused epilogues)
# ---------------------------------------------------------------------------
def linear_fp16(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """``x @ w^T`` with fp32 accumulation, rounded to fp16 (returned as fp32).

    dit_source_oracle.py:93-96 (``linear``: F.linear in fp32, cast to the input
    dtype) -- the reference's LinearExecutor output (LinearExecutor.swift:79-)
    is fp16.  ``x`` is ``[m, k]``, ``w`` the ``[n, k]`` (out, in) weight.
    """
    xf = np.asarray(x, dtype=np.float32)
    wf = np.asarray(w, dtype=np.float32)
    return to_fp16_storage(xf @ wf.T)


def qkv_norm_projection(x, w, *, q_cols: int, k_cols: int, qk_norm: str = "rms_rope",
                        q_norm_weight=None, k_norm_weight=None, rope_table=None,
                        tokens: int | None = None, eps: float = EPS) -> np.ndarray:
    """The fused q|k|v projection: ``y = linear_fp16(x, w)``; the q heads
    (columns ``[0, q_cols)``) and k heads (``[q_cols, q_cols + k_cols)``), 128
    wide, are RMS-normalised with fp32 statistics (``rms_norm_heads``) and, for
    ``"rms_rope"``, rotated (``apply_split_half_rope``, table row = row % tokens);
    the rest (v) is ``y``.  DiTBlockExecutor.swift:1097-1131 then
    AnimaKernels.metal:660-729 (dit_source_oracle.py:262-272).  fp32 result,
    to be compared after fp16 storage.
    """
    y = linear_fp16(x, w)
    m = y.shape[0]
    tokens = m if tokens is None else tokens
    out = y.copy()
    for c0, c1, wt in ((0, q_cols, q_norm_weight), (q_cols, q_cols + k_cols, k_norm_weight)):
        if c1 <= c0:
            continue
        h = y[:, c0:c1].reshape(m // tokens, tokens, (c1 - c0) // 128, 128)
        h = rms_norm_heads(h, wt, eps)
        if qk_norm == "rms_rope":
            h = apply_split_half_rope(h, rope_table)
        out[:, c0:c1] = h.reshape(m, c1 - c0)
    return out


def gate_add_projection(residual, x, w, gate, *, tokens: int) -> np.ndarray:
    """``residual + float(linear_fp16(x, w)) * gate[row // tokens]`` in fp32:
    the out-projection then gate_add_half_f32 (AnimaKernels.metal:624-634,
    DiTBlockExecutor.swift:1223-1236; dit_source_oracle.py:317
    ``x + gate * out``)."""
    branch = linear_fp16(x, w)
    g = np.asarray(gate, dtype=np.float32)
    rows = np.arange(branch.shape[0]) // tokens
    return (np.asarray(residual, dtype=np.float32) + branch * g[rows]).astype(np.float32)


# ---------------------------------------------------------------------------
# Quantized (W4 / W8) projection weights
# ---------------------------------------------------------------------------
QUANT_GROUP = 64


def dequant_to_half(packed: np.ndarray, scale: np.ndarray, zero: np.ndarray, *, bits: int,
                    k: int) -> np.ndarray:
    """Decode W8 / W4 codes to fp16 (returned as float16).

    ``packed`` is ``[rows][>= k]`` bytes (W8) or ``[rows][>= ceil(k / 2)]``
    (W4: column ``2j`` in the low nibble of byte ``j``, ``2j + 1`` in the high
    nibble); ``scale`` / ``zero`` are fp16 ``[rows][ceil(k / 64)]``, the groups of
    64 columns restarting at every row.  value = ``q * scale + zero`` in fp32
    (one rounding after the multiply, one after the add) then rounded to fp16:
    scripts/animapk_cuda/quant.py:32-76 (``q * sg + zg``) and
    AnimaKernels.metal:19-67 (``half(float(q) * float(sc) + float(ze))``).
    """
    packed = np.asarray(packed, dtype=np.uint8)
    rows = packed.shape[0]
    if bits == 4:
        q = np.empty((rows, 2 * packed.shape[1]), dtype=np.uint8)
        q[:, 0::2] = packed & 0x0F
        q[:, 1::2] = packed >> 4
        q = q[:, :k]
    elif bits == 8:
        q = packed[:, :k]
    else:
        raise ValueError("bits must be 4 or 8")
    g = np.arange(k) // QUANT_GROUP
    sc = np.asarray(scale, dtype=np.float16).astype(np.float32)[:, g]
    ze = np.asarray(zero, dtype=np.float16).astype(np.float32)[:, g]
    prod = (q.astype(np.float32) * sc).astype(np.float32)
    return (prod + ze).astype(np.float32).astype(np.float16)


# ---------------------------------------------------------------------------
# Score-health probe
# ---------------------------------------------------------------------------
PROBE_NAN, PROBE_POS_INF, PROBE_NEG_INF, PROBE_HALF_OVERFLOW = 1, 2, 4, 8


def score_health(q: np.ndarray, k: np.ndarray, *, scale: float | None = None, causal: bool = False,
                 kv_valid_len=None) -> tuple[int, float, int]:
    """(flags, max |score|, first flagged key) of the scaled scores
    ``scale * q.k`` over each row's unmasked keys, as the reference's
    attention_softmax_rows_probe records them (AnimaKernels.metal:1738-1830):
    NaN, +Inf, -Inf, and |score| > 65504 flag a score; the magnitude is the
    largest |score| among the finite ones; the index is the smallest flagged
    key column (0xFFFFFFFF when none).  Scores here are fp32 (the reference
    rounds them to fp16 first).  ``q``/``k`` are ``[B, S, H, D]`` (GQA by
    ``gqa_kv_head``)."""
    qf = np.asarray(q, dtype=np.float32)
    kf = np.asarray(k, dtype=np.float32)
    b, sq, hq, d = qf.shape
    sk, hkv = kf.shape[1], kf.shape[2]
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    flags, max_abs, first = 0, 0.0, 0xFFFFFFFF
    with np.errstate(invalid="ignore", over="ignore"):
        for bi in range(b):
            valid = sk if kv_valid_len is None else int(kv_valid_len[bi] if np.ndim(kv_valid_len) else kv_valid_len)
            for h in range(hq):
                kh = gqa_kv_head(h, hq, hkv)
                s = (qf[bi, :, h, :] @ kf[bi, :, kh, :].T).astype(np.float32)   # [sq, sk] raw q.k
                mask = np.broadcast_to(np.arange(sk)[None, :] < valid, s.shape)
                if causal:
                    mask = mask & (np.arange(sk)[None, :] <= np.arange(sq)[:, None])
                sv = s[mask]
                cols = np.broadcast_to(np.arange(sk)[None, :], s.shape)[mask]
                nan = np.isnan(sv)
                pinf = np.isposinf(sv)
                ninf = np.isneginf(sv)
                finite = np.isfinite(sv)
                a = np.abs(sv[finite]) * np.float32(scale)
                over = np.zeros_like(sv, dtype=bool)
                over[finite] = a > 65504.0
                flags |= (PROBE_NAN if nan.any() else 0) | (PROBE_POS_INF if pinf.any() else 0) | \
                    (PROBE_NEG_INF if ninf.any() else 0) | (PROBE_HALF_OVERFLOW if over.any() else 0)
                if a.size:
                    max_abs = max(max_abs, float(a.max()))
                bad = nan | pinf | ninf | over
                if bad.any():
                    first = min(first, int(cols[bad].min()))
    return flags, max_abs, first
