"""Host mirror of the cross-attention K/V cache (``animaxs_cross_kv_cache_*``
in ``include/animaxs_attn.h``): the reference's ``CrossKVCache``
(AnimaXS/Runtime/Metal/DiTBlockExecutor.swift:19-43) and its use by the DiT
block (:1105-1161).

The cross-attention K/V of each block depend only on the LLM-adapter context,
so they are computed once per generation (projected, K RMS-normalised) and
reused by the other Euler steps.  A hit costs nothing here: attention reads
the cached block in place (``qk_norm_targets="q"``), where the reference
blits it back into its scratch buffers.  The reference's names are kept:
``tensor_bytes``, ``block_stride``, ``block_count``, ``k_offset``,
``v_offset``, ``is_ready``, ``mark_ready``.  Like the reference's cache it
belongs to one generation; :meth:`reset` starts the next.
"""

from __future__ import annotations

import ctypes

from . import _lib
from .executor import AttentionExecutor, _stream_handle


class CrossKVCache:
    """``blocks`` blocks of ``[batch][tokens][K | V]`` fp16 rows on the
    executor's device; ``k(block)`` / ``v(block)`` are ``[batch, tokens,
    kv_heads, head_dim]`` views for :meth:`AttentionExecutor.attention`."""

    def __init__(self, executor: AttentionExecutor, blocks: int = 28, batch: int = 1, tokens: int = 512,
                 kv_heads: int = 16, head_dim: int = 128):
        import torch
        self.ex = executor
        self._lib = executor._lib
        self.blocks, self.batch, self.tokens = int(blocks), int(batch), int(tokens)
        self.kv_heads, self.head_dim = int(kv_heads), int(head_dim)
        nbytes = ctypes.c_int64()
        rc = self._lib.animaxs_cross_kv_cache_bytes(self.blocks, self.batch, self.tokens, self.kv_heads,
                                                    self.head_dim, ctypes.byref(nbytes))
        _lib.raise_for(rc, "invalid cross-K/V cache shape (head_dim 64 or 128, positive sizes)")
        # The memory is a torch allocation so that the blocks can be viewed as tensors.
        self.buffer = torch.empty(nbytes.value // 2, dtype=torch.float16,
                                  device=torch.device("cuda", executor.device))
        handle = ctypes.c_void_p()
        rc = self._lib.animaxs_cross_kv_cache_create(executor.handle, self.blocks, self.batch, self.tokens,
                                                     self.kv_heads, self.head_dim, self.buffer.data_ptr(),
                                                     nbytes.value, ctypes.byref(handle))
        executor._check(rc)
        self._h = handle

    # -- the reference's layout constants (bytes) --------------------------
    @property
    def block_count(self) -> int:
        return self.blocks

    @property
    def tensor_bytes(self) -> int:
        """Bytes of one block's K (or V) for all tokens and images."""
        return self.batch * self.tokens * self.kv_heads * self.head_dim * 2

    @property
    def block_stride(self) -> int:
        return 2 * self.tensor_bytes

    def k_offset(self, block: int) -> int:
        """Byte offset of the block's first K row (rows are 2 x kv_heads x head_dim fp16 apart)."""
        return block * self.block_stride

    def v_offset(self, block: int) -> int:
        """Byte offset of the block's first V row (inside the first K|V row)."""
        return self.k_offset(block) + self.kv_heads * self.head_dim * 2

    def is_ready(self, block: int) -> bool:
        r = ctypes.c_int()
        rc = self._lib.animaxs_cross_kv_cache_block(self._h, block, None, None, None, None, ctypes.byref(r))
        _lib.raise_for(rc, f"cross-K/V cache block {block} out of range")
        return bool(r.value)

    def mark_ready(self, block: int, ready: bool = True) -> None:
        self.ex._check(self._lib.animaxs_cross_kv_cache_mark_ready(self._h, block, 1 if ready else 0))

    def reset(self) -> None:
        self.ex._check(self._lib.animaxs_cross_kv_cache_reset(self._h))

    # -- views ---------------------------------------------------------------
    def _view(self, block: int, which: int):
        row = 2 * self.kv_heads * self.head_dim
        base = block * self.batch * self.tokens * row + which * self.kv_heads * self.head_dim
        return self.buffer.as_strided((self.batch, self.tokens, self.kv_heads, self.head_dim),
                                      (self.tokens * row, row, self.head_dim, 1), base)

    def k(self, block: int):
        """The block's (normalised) K, [batch, tokens, kv_heads, head_dim]."""
        return self._view(block, 0)

    def v(self, block: int):
        return self._view(block, 1)

    # -- filling ---------------------------------------------------------------
    def fill(self, block: int, k, v, *, k_norm: bool = True, k_norm_weight=None, eps: float = 1e-6,
             stream=None) -> None:
        """Store projected ``k``/``v`` ([batch, tokens, kv_heads, head_dim]
        fp16, any token / batch stride, rows contiguous); K RMS-normalised by
        the attention prologue's kernel unless ``k_norm`` is False."""
        import torch
        for t in (k, v):
            if t.shape != (self.batch, self.tokens, self.kv_heads, self.head_dim) or t.stride(3) != 1 \
                    or t.stride(2) != self.head_dim:
                raise _lib.AttentionValidationError(
                    _lib.ERR_INVALID_ARG, "k and v must be [batch, tokens, kv_heads, head_dim] with packed heads")
        if stream is None:
            stream = torch.cuda.current_stream(k.device)
        w = None if k_norm_weight is None else k_norm_weight.data_ptr()
        rc = self._lib.animaxs_cross_kv_cache_fill(self._h, block, k.data_ptr(), k.stride(1), k.stride(0),
                                                   v.data_ptr(), v.stride(1), v.stride(0), 1 if k_norm else 0,
                                                   w, eps, _stream_handle(stream))
        self.ex._check(rc)

    def project(self, block: int, context, w_kv, *, k_norm_weight=None, eps: float = 1e-6,
                stream=None) -> None:
        """Project the adapter ``context`` ([batch x tokens, context_dim]) with
        the stacked cross weights ``w_kv`` ([2 x kv_heads x 128, context_dim]:
        W_k rows then W_v rows) into the block, K RMS-normalised in the GEMM
        epilogue (the reference's miss path, DiTBlockExecutor.swift:1123-1160)."""
        import torch
        if context.stride(1) != 1 or w_kv.stride(1) != 1:
            raise _lib.AttentionValidationError(_lib.ERR_INVALID_ARG, "context and w_kv need contiguous rows")
        if stream is None:
            stream = torch.cuda.current_stream(context.device)
        w = None if k_norm_weight is None else k_norm_weight.data_ptr()
        rc = self._lib.animaxs_cross_kv_cache_project(self._h, block, context.data_ptr(), context.stride(0),
                                                      context.shape[1], w_kv.data_ptr(), w_kv.stride(0), w,
                                                      eps, _stream_handle(stream))
        self.ex._check(rc)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.animaxs_cross_kv_cache_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
