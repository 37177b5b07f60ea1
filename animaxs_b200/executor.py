"""Host-side mirror of the reference's ``AttentionExecutor`` over the C ABI.

The reference operator is the Swift class ``AttentionExecutor``
(``AnimaXS/Runtime/Metal/AttentionExecutor.swift:77-848``).  This class keeps
its argument names (``query/queryOffset/key/.../heads/queryCount/keyCount/
headDim/keyValueHeads/causal/layout`` in snake_case), its two layouts
(``AttentionInputLayout.headMajor`` / ``.tokenMajor(tokenStride:)``), its
scratch query (``maximumScoreScratchBytes``) and its error behaviour
(``AnimapkError.validation`` -> :class:`AttentionValidationError` with the
reference's messages).  ``encode`` enqueues on a CUDA stream (the reference
encodes into an ``MTLCommandBuffer``); ``execute`` runs and waits (the
reference's ``execute ... async throws``).

Buffers are device allocations given as objects with ``data_ptr()`` plus
``numel()``/``element_size()`` (torch tensors) or :class:`DeviceBuffer`;
offsets are in bytes, as in the reference.

Extensions beyond the reference interface (keyword-only): the fused q/k
``qk_norm`` prologue (the reference encodes it as separate kernels in front of
the attention, ``DiTBlockExecutor.swift:1139-1172``), key-padding
``kv_valid_len`` and an explicit ``scale``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import (AttentionValidationError, AttnDesc, QK_NONE, QK_RMS, QK_RMS_ROPE, lib,
                   raise_for)

NUMERICS = ("legacy", "fp32ScoresAndSoftmax", "bf16_compute")
# animaxs_numerics
_NUMERICS = {"legacy": _lib.NUMERICS_LEGACY, "fp32ScoresAndSoftmax": _lib.NUMERICS_FP32,
             "bf16_compute": _lib.NUMERICS_BF16}
BACKENDS = ("legacyHeadMajorMPS", "stridedTokenMajorMPS", "streamingMPS", "metalFlash")
_QK = {"none": QK_NONE, "rms": QK_RMS, "rms_rope": QK_RMS_ROPE}
# animaxs_qk_norm_targets: which of q and k the qk_norm mode applies to.
_QK_TARGETS = {"both": 0, "q": 1, "k": 2}


@dataclass(frozen=True)
class DeviceBuffer:
    """A raw device allocation (pointer + length in bytes), the MTLBuffer stand-in."""
    ptr: int
    length: int


@dataclass(frozen=True)
class AttentionInputLayout:
    """``.headMajor`` ([heads, rows, headDim]) or ``.tokenMajor(tokenStride:)``."""
    token_stride: int | None = None

    @property
    def is_token_major(self) -> bool:
        return self.token_stride is not None

    @staticmethod
    def token_major(token_stride: int) -> "AttentionInputLayout":
        return AttentionInputLayout(int(token_stride))


AttentionInputLayout.head_major = AttentionInputLayout(None)


def _ptr_len(buf):
    if isinstance(buf, DeviceBuffer):
        return buf.ptr, buf.length
    if hasattr(buf, "data_ptr"):
        if hasattr(buf, "is_cuda") and not buf.is_cuda:
            raise AttentionValidationError(_lib.ERR_INVALID_ARG, "attention buffers must be device memory")
        return int(buf.data_ptr()), int(buf.numel() * buf.element_size())
    raise TypeError(f"unsupported buffer type {type(buf)!r}")


def _stream_handle(stream):
    if stream is None:
        return None
    if hasattr(stream, "cuda_stream"):
        return ctypes.c_void_p(stream.cuda_stream)
    return ctypes.c_void_p(int(stream))


class AttentionExecutor:
    """Query-tiled scaled dot-product attention on B200 (tcgen05 flash kernel).

    Like the reference, an executor is NOT reentrant: it owns scratch memory.
    """

    default_tile_rows = 128

    def __init__(self, device: int = 0, tile_rows: int = default_tile_rows,
                 numerics: str = "legacy", layout: AttentionInputLayout = AttentionInputLayout.head_major,
                 attention_backend: str = "legacyHeadMajorMPS"):
        if tile_rows <= 0:
            raise AttentionValidationError(_lib.ERR_INVALID_ARG, "tileRows must be positive")
        if numerics not in NUMERICS:
            raise AttentionValidationError(_lib.ERR_INVALID_ARG, f"unknown numerics {numerics!r}")
        if attention_backend not in BACKENDS:
            raise AttentionValidationError(_lib.ERR_INVALID_ARG, f"unknown backend {attention_backend!r}")
        self.device = int(device)
        self.tile_rows = int(tile_rows)
        self.numerics = numerics
        self.layout = layout
        self.attention_backend = attention_backend
        self._lib = lib()
        ctx = ctypes.c_void_p()
        rc = self._lib.animaxs_attn_create(self.device, ctypes.byref(ctx))
        raise_for(rc, f"no sm_100 device {device} (animaxs_attn_create -> {rc})")
        self._ctx = ctx
        self._desc_cache = {}

    # -- lifetime ---------------------------------------------------------
    def close(self):
        if getattr(self, "_ctx", None):
            self._lib.animaxs_attn_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._ctx

    def last_error(self) -> str:
        return self._lib.animaxs_attn_last_error(self._ctx).decode()

    def _check(self, rc: int):
        raise_for(rc, self.last_error())

    # -- reference interface ---------------------------------------------
    def maximum_score_scratch_bytes(self, key_count: int, query_count: int | None = None) -> int:
        """AttentionExecutor.swift:112-120: bytes of the fp16 (fp32 for the
        fp32 numerics) score tile ``[min(tileRows, queryCount), keyCount]``
        that the reference keeps.  The flash kernel keeps scores in TMEM and
        needs none of it; the number is reported for interface parity."""
        if key_count <= 0:
            raise AttentionValidationError(_lib.ERR_INVALID_ARG, "attention key count must be positive")
        tile = self.tile_rows if query_count is None else min(self.tile_rows, query_count)
        elem = 2 if self.numerics == "legacy" else 4
        return tile * key_count * elem

    @property
    def attention_query_tiles(self) -> int:
        """(head, 128-row tile) units executed (MetricsCollector.recordAttentionQueryTile)."""
        v = ctypes.c_int64()
        self._check(self._lib.animaxs_attn_query_tiles(self._ctx, ctypes.byref(v)))
        return v.value

    def set_score_probe(self, probe) -> None:
        """Record the health of every following call's scores into ``probe``
        (a :class:`~animaxs_b200.probe.ScoreProbe`, or None to stop); the
        ``monitor``/``probe`` pair of the reference's executor."""
        ptr = None if probe is None else probe.data_ptr()
        self._check(self._lib.animaxs_attn_set_score_probe(self._ctx, ptr))
        self._score_probe = probe

    def set_kernel_timing(self, enable: bool):
        """Bracket every flash-kernel launch with CUDA events (see kernel_timing)."""
        self._check(self._lib.animaxs_attn_set_kernel_timing(self._ctx, 1 if enable else 0))

    def kernel_timing(self):
        """(launches, total_ms, max_ms) of the flash kernel since the last read."""
        n, tot, mx = ctypes.c_int64(), ctypes.c_double(), ctypes.c_double()
        self._check(self._lib.animaxs_attn_kernel_timing(self._ctx, ctypes.byref(n), ctypes.byref(tot),
                                                         ctypes.byref(mx)))
        return n.value, tot.value, mx.value

    def make_desc(self, *, heads, query_count, key_count, head_dim, key_value_heads=None,
                  causal=False, layout=None, qk_norm="none", q_norm_weight=None,
                  k_norm_weight=None, rope_table=None, eps=1e-6, kv_valid_len=None,
                  kv_valid_lens=None, scale=None, batch=1, lengths=(0, 0, 0, 0),
                  qk_norm_targets="both") -> AttnDesc:
        kv_heads = heads if key_value_heads is None else key_value_heads
        layout = self.layout if layout is None else layout
        if layout.is_token_major:
            ts = layout.token_stride
            if not (ts > 0 and head_dim <= ts and ts % max(head_dim, 1) == 0
                    and heads * head_dim == ts and kv_heads == heads):
                raise AttentionValidationError(
                    _lib.ERR_INVALID_ARG,
                    "token-major attention requires tokenStride == heads * headDim and keyValueHeads == heads")
            if self.numerics == "fp32ScoresAndSoftmax":
                raise AttentionValidationError(
                    _lib.ERR_UNSUPPORTED,
                    "strided token-major attention does not support fp32ScoresAndSoftmax; select baseline numerics")
        if self.numerics == "bf16_compute":
            raise AttentionValidationError(
                _lib.ERR_UNSUPPORTED,
                "bf16Compute numerics emulates Apple5 BF16 rounding and is not built for B200")
        d = AttnDesc()
        self._lib.animaxs_attn_desc_init(ctypes.byref(d), batch, heads, kv_heads, query_count,
                                         key_count, head_dim)
        d.numerics = _NUMERICS[self.numerics]
        if layout.is_token_major:
            ts = layout.token_stride
            d.q_tok_stride = d.o_tok_stride = ts
            d.k_tok_stride = d.v_tok_stride = ts
            d.q_head_stride = d.k_head_stride = d.v_head_stride = d.o_head_stride = head_dim
            d.q_batch_stride = d.o_batch_stride = query_count * ts
            d.k_batch_stride = d.v_batch_stride = key_count * ts
        else:
            d.q_tok_stride = d.k_tok_stride = d.v_tok_stride = d.o_tok_stride = head_dim
            d.q_head_stride = d.o_head_stride = query_count * head_dim
            d.k_head_stride = d.v_head_stride = key_count * head_dim
            d.q_batch_stride = d.o_batch_stride = heads * query_count * head_dim
            d.k_batch_stride = d.v_batch_stride = kv_heads * key_count * head_dim
        d.causal = 1 if causal else 0
        d.kv_valid_len = 0 if kv_valid_len is None else int(kv_valid_len)
        d.kv_valid_lens = None if kv_valid_lens is None else _ptr_len(kv_valid_lens)[0]
        d.scale = 0.0 if scale is None else float(scale)
        if qk_norm not in _QK:
            raise AttentionValidationError(_lib.ERR_INVALID_ARG, f"unknown qk_norm {qk_norm!r}")
        d.qk_norm = _QK[qk_norm]
        if qk_norm_targets not in _QK_TARGETS:
            raise AttentionValidationError(_lib.ERR_INVALID_ARG,
                                           f"unknown qk_norm_targets {qk_norm_targets!r}")
        d.qk_norm_targets = _QK_TARGETS[qk_norm_targets]
        d.eps = float(eps)
        d.q_norm_weight = None if q_norm_weight is None else _ptr_len(q_norm_weight)[0]
        d.k_norm_weight = None if k_norm_weight is None else _ptr_len(k_norm_weight)[0]
        if rope_table is not None:
            ptr, length = _ptr_len(rope_table)
            d.rope_table = ptr
            d.rope_rows = length // (head_dim // 2 * 4 * 4)
        d.q_bytes, d.k_bytes, d.v_bytes, d.o_bytes = lengths
        return d

    def encode(self, stream, query, key, value, output, *, heads: int, query_count: int,
               key_count: int, head_dim: int, query_offset: int = 0, key_offset: int = 0,
               value_offset: int = 0, output_offset: int = 0, key_value_heads: int | None = None,
               causal: bool = False, layout: AttentionInputLayout | None = None, probe=None, **ext):
        """AttentionExecutor.encode (AttentionExecutor.swift:122-302): enqueue on ``stream``.
        ``probe`` (a :class:`~animaxs_b200.probe.ScoreProbe`) records this
        call's score health, as the reference's ``probe:`` argument."""
        offsets = (query_offset, key_offset, value_offset, output_offset)
        if min(offsets) < 0:
            raise AttentionValidationError(_lib.ERR_INVALID_ARG,
                                           "invalid attention shape, offset, or causal dimensions")
        ptrs, lens = [], []
        for buf, off in zip((query, key, value, output), offsets):
            p, n = _ptr_len(buf)
            ptrs.append(p + off)
            lens.append(max(n - off, 1) if off <= n else 1)
        d = self.make_desc(heads=heads, query_count=query_count, key_count=key_count,
                           head_dim=head_dim, key_value_heads=key_value_heads, causal=causal,
                           layout=layout, lengths=tuple(lens), **ext)
        outer = getattr(self, "_score_probe", None)
        if probe is not None:
            self._check(self._lib.animaxs_attn_set_score_probe(self._ctx, probe.data_ptr()))
        try:
            rc = self._lib.animaxs_attn_forward(self._ctx, ctypes.byref(d), *[ctypes.c_void_p(p) for p in ptrs],
                                                _stream_handle(stream))
        finally:
            if probe is not None:  # back to the probe set with set_score_probe, if any
                self._lib.animaxs_attn_set_score_probe(self._ctx, None if outer is None else outer.data_ptr())
        self._check(rc)

    def strided_desc(self, q, k, v, out, *, causal=False, qk_norm="none", rope_table=None,
                     q_norm_weight=None, k_norm_weight=None, eps=1e-6, kv_valid_len=None,
                     kv_valid_lens=None, scale=None, qk_norm_targets="both") -> AttnDesc:
        """Descriptor for ``[B, S, H, D]`` tensors (D 64, 128, 256 or 384) with arbitrary strides (cached)."""
        key = (q.shape, k.shape, q.stride(), k.stride(), v.stride(), out.stride(), causal, qk_norm,
               None if rope_table is None else (rope_table.data_ptr(), rope_table.numel()),
               None if q_norm_weight is None else q_norm_weight.data_ptr(),
               None if k_norm_weight is None else k_norm_weight.data_ptr(), eps, kv_valid_len,
               None if kv_valid_lens is None else kv_valid_lens.data_ptr(), scale, qk_norm_targets)
        desc = self._desc_cache.get(key)
        if desc is None:
            b, sq, h, d = q.shape
            sk, hkv = k.shape[1], k.shape[2]
            desc = self.make_desc(heads=h, query_count=sq, key_count=sk, head_dim=d,
                                  key_value_heads=hkv, causal=causal,
                                  layout=AttentionInputLayout.head_major, qk_norm=qk_norm,
                                  q_norm_weight=q_norm_weight, k_norm_weight=k_norm_weight,
                                  rope_table=rope_table, eps=eps, kv_valid_len=kv_valid_len,
                                  kv_valid_lens=kv_valid_lens, scale=scale, batch=b,
                                  qk_norm_targets=qk_norm_targets)
            for name, t in (("q", q), ("k", k), ("v", v), ("o", out)):
                sb, st, sh, sd = t.stride()
                if sd != 1:
                    raise AttentionValidationError(_lib.ERR_INVALID_ARG, "head_dim must be contiguous")
                setattr(desc, f"{name}_batch_stride", sb)
                setattr(desc, f"{name}_tok_stride", st)
                setattr(desc, f"{name}_head_stride", sh)
            if len(self._desc_cache) > 256:
                self._desc_cache.clear()
            self._desc_cache[key] = desc
        return desc

    def attention(self, q, k, v, out=None, *, stream=None, **kw):
        """Strided entry: ``q``/``out`` are ``[B, Sq, H, D]`` and ``k``/``v``
        ``[B, Sk, Hkv, D]`` fp16 device tensors, D 64, 128, 256 or 384, with ANY strides (token-major,
        head-major views, batch gaps).  Keywords: ``causal``, ``qk_norm``
        (``"none"``/``"rms"``/``"rms_rope"``), ``qk_norm_targets`` (``"both"``, or
        ``"q"`` when k is already normalised, e.g. a cached cross K), ``rope_table``, ``q_norm_weight``,
        ``k_norm_weight``, ``eps``, ``kv_valid_len``, ``kv_valid_lens``, ``scale``.
        Enqueues on ``stream`` (default: the current torch stream); returns ``out``."""
        import torch
        if out is None:
            out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        desc = self.strided_desc(q, k, v, out, **kw)
        if stream is None:
            stream = torch.cuda.current_stream(q.device)
        rc = self._lib.animaxs_attn_forward(self._ctx, ctypes.byref(desc), q.data_ptr(), k.data_ptr(),
                                            v.data_ptr(), out.data_ptr(), _stream_handle(stream))
        self._check(rc)
        return out

    def execute(self, query, key, value, output, **kw):
        """AttentionExecutor.execute (AttentionExecutor.swift:751-776): run and wait."""
        import torch
        stream = torch.cuda.current_stream(self.device)
        self.encode(stream, query, key, value, output, **kw)
        self.synchronize(stream)

    def synchronize(self, stream=None):
        self._check(self._lib.animaxs_attn_synchronize(self._ctx, _stream_handle(stream)))

    # -- standalone qk prologues (AnimaKernels.metal:660-729) -------------
    def rms_rope_split_half(self, stream, inp, out, weight, rope_table, *, tokens, heads,
                            head_dim=128, row_stride=0, eps=1e-6):
        w = None if weight is None else _ptr_len(weight)[0]
        rc = self._lib.animaxs_rms_rope_split_half(
            self._ctx, _ptr_len(inp)[0], _ptr_len(out)[0], w, _ptr_len(rope_table)[0],
            tokens, heads, head_dim, row_stride, eps, _stream_handle(stream))
        self._check(rc)

    def rmsnorm_heads_half(self, stream, inp, out, weight, *, tokens, heads, head_dim=128,
                           row_stride=0, eps=1e-6):
        w = None if weight is None else _ptr_len(weight)[0]
        rc = self._lib.animaxs_rmsnorm_heads_half(
            self._ctx, _ptr_len(inp)[0], _ptr_len(out)[0], w, tokens, heads, head_dim,
            row_stride, eps, _stream_handle(stream))
        self._check(rc)


class DitRoPE:
    """DitRoPE.generate(T:H:W:) (AnimaXS/Runtime/Text/DitRoPE.swift:58-107) via the C helper."""
    head_dim = 128
    num_freqs = 64

    @staticmethod
    def generate(T: int = 1, H: int = 32, W: int = 32) -> np.ndarray:
        out = np.empty(T * H * W * 64 * 4, dtype=np.float32)
        rc = lib().animaxs_rope3d_table(T, H, W, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        raise_for(rc, "invalid rope grid")
        return out


def qwen_rope(tokens: int, theta: float = 1.0e6, head_dim: int = 128) -> np.ndarray:
    """QwenEncoderMetal.makeRope(tokens:) (QwenEncoderMetal.swift:126-142)."""
    out = np.empty(tokens * head_dim // 2 * 4, dtype=np.float32)
    rc = lib().animaxs_rope1d_table(tokens, head_dim, theta,
                                    out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    raise_for(rc, "invalid rope length")
    return out


def adapter_rope(tokens: int) -> np.ndarray:
    """LLMAdapterMetal.makeRope(tokens:) (LLMAdapterMetal.swift:162-178): the
    LLM adapter's [tokens][32][2][2] table (theta 1e4, 64-wide heads) for
    ``qk_norm="rms_rope"`` on head_dim-64 calls."""
    return qwen_rope(tokens, theta=1.0e4, head_dim=64)


class GqaHeadMapping:
    """Q head h reads KV head h / (heads / kvHeads) (AttentionExecutor.swift:222)."""

    @staticmethod
    def kv_head(query_head: int, query_heads: int, kv_heads: int) -> int:
        r = lib().animaxs_gqa_kv_head(query_head, query_heads, kv_heads)
        if r < 0:
            raise AttentionValidationError(r, "query heads must be divisible by kv heads")
        return r
