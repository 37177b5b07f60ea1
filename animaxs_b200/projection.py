"""Host mirror of the fused attention projections (``animaxs_proj_*`` in
``include/animaxs_attn.h``): the reference's ``LinearExecutor.encode``
(LinearExecutor.swift:79-) for the q/k/v and out projections, with the
elementwise step each is followed by in DiTBlockExecutor.swift:1097-1131 /
1223-1236 fused into the GEMM epilogue.

``x`` is ``[m, k]`` fp16 (rows = images x tokens, any row stride), ``w`` the
reference's ``[n, k]`` (out, in) fp16 weight or a :class:`QuantizedWeight`
(W8 / W4 codes, decoded on the device before the GEMM).  Shares the context
(and so the stream and error state) of an :class:`AttentionExecutor`.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _lib
from ._lib import (PROJ_GATE_ADD, PROJ_QKV_NORM, PROJ_STORE, ProjDesc, QK_RMS, QK_RMS_ROPE, WEIGHT_W4,
                   WEIGHT_W8)
from .executor import AttentionExecutor, _stream_handle


@dataclass
class QuantizedWeight:
    """A W8 / W4 weight in the reference's pack layout (QuantizedLinearWeightBuffers,
    LinearExecutor.swift:12-40): ``packed`` uint8 ``[n][>= k]`` (W8) or
    ``[n][>= ceil(k / 2)]`` (W4, column ``2j`` in the low nibble of byte ``j``),
    ``scale`` / ``zero`` fp16 ``[n][ceil(k / 64)]``; all on the device."""
    packed: object
    scale: object
    zero: object
    bits: int
    k: int

    @property
    def shape(self):
        return (self.packed.shape[0], self.k)


class ProjectionExecutor:
    def __init__(self, executor: AttentionExecutor):
        self.ex = executor
        self._lib = executor._lib

    def _desc(self, x, w, out, epilogue, tokens):
        m, k = x.shape
        n = w.shape[0]
        quant = isinstance(w, QuantizedWeight)
        wrow = w.packed if quant else w
        if w.shape[1] != k or x.stride(1) != 1 or wrow.stride(1) != 1 or out.stride(1) != 1:
            raise _lib.AttentionValidationError(_lib.ERR_INVALID_ARG,
                                                "x [m, k], w [n, k] and out [m, n] need contiguous rows")
        d = ProjDesc()
        self._lib.animaxs_proj_desc_init(ctypes.byref(d), m, n, k, epilogue)
        d.x_stride, d.out_stride = x.stride(0), out.stride(0)
        d.w_stride = k if quant else w.stride(0)
        if quant:
            if w.bits not in (4, 8):
                raise _lib.AttentionValidationError(_lib.ERR_INVALID_ARG, "bits must be 4 or 8")
            d.w_storage = WEIGHT_W4 if w.bits == 4 else WEIGHT_W8
            d.w_scale, d.w_zero = w.scale.data_ptr(), w.zero.data_ptr()
            d.w_packed_stride = w.packed.stride(0)
        d.tokens = m if tokens is None else int(tokens)
        return d

    def dequant(self, w: QuantizedWeight, out=None, *, stream=None):
        """fp16 ``[n, k]`` decode of ``w`` (dequant_w8_to_half / dequant_w4_to_half,
        AnimaKernels.metal:19-67)."""
        import torch
        n = w.packed.shape[0]
        if out is None:
            out = torch.empty(n, w.k, dtype=torch.float16, device=w.packed.device)
        if stream is None:
            stream = torch.cuda.current_stream(w.packed.device)
        if w.packed.stride(1) != 1 or out.stride(1) != 1:
            raise _lib.AttentionValidationError(_lib.ERR_INVALID_ARG, "packed and out need contiguous rows")
        rc = self._lib.animaxs_dequant_to_half(self.ex.handle, int(w.bits), w.packed.data_ptr(),
                                               w.scale.data_ptr(), w.zero.data_ptr(), out.data_ptr(), n,
                                               int(w.k), w.packed.stride(0), out.stride(0),
                                               _stream_handle(stream))
        self.ex._check(rc)
        return out

    def _run(self, d, x, w, out, stream):
        import torch
        if stream is None:
            stream = torch.cuda.current_stream(x.device)
        wptr = (w.packed if isinstance(w, QuantizedWeight) else w).data_ptr()
        rc = self._lib.animaxs_proj_forward(self.ex.handle, ctypes.byref(d), x.data_ptr(), wptr,
                                            out.data_ptr(), _stream_handle(stream))
        self.ex._check(rc)
        return out

    def linear(self, x, w, out=None, *, stream=None):
        """``out = fp16(x w^T)`` (LinearExecutor.encode)."""
        import torch
        if out is None:
            out = torch.empty(x.shape[0], w.shape[0], dtype=torch.float16, device=x.device)
        return self._run(self._desc(x, w, out, PROJ_STORE, None), x, w, out, stream)

    def qkv(self, x, w, out=None, *, q_cols: int, k_cols: int, qk_norm: str = "rms_rope",
            q_norm_weight=None, k_norm_weight=None, rope_table=None, tokens: int | None = None,
            eps: float = 1e-6, stream=None):
        """Fused q|k|v projection: ``fp16(x w^T)`` with the q heads (columns
        ``[0, q_cols)``) and k heads (``[q_cols, q_cols + k_cols)``) RMS-normalised
        and, for ``qk_norm="rms_rope"``, rotated with ``rope_table`` (row =
        row % tokens).  The result's column ranges are the q, k, v inputs of
        :meth:`AttentionExecutor.attention` with ``qk_norm="none"``."""
        import torch
        if out is None:
            out = torch.empty(x.shape[0], w.shape[0], dtype=torch.float16, device=x.device)
        d = self._desc(x, w, out, PROJ_QKV_NORM, tokens)
        if qk_norm not in ("rms", "rms_rope"):
            raise _lib.AttentionValidationError(_lib.ERR_INVALID_ARG, f"unknown qk_norm {qk_norm!r}")
        d.qk_norm = QK_RMS_ROPE if qk_norm == "rms_rope" else QK_RMS
        d.q_cols, d.k_cols = int(q_cols), int(k_cols)
        d.q_norm_weight = None if q_norm_weight is None else q_norm_weight.data_ptr()
        d.k_norm_weight = None if k_norm_weight is None else k_norm_weight.data_ptr()
        if rope_table is not None:
            d.rope_table = rope_table.data_ptr()
            d.rope_rows = rope_table.numel() // (64 * 4)
        d.eps = float(eps)
        return self._run(d, x, w, out, stream)

    def out_gate_add(self, x, w, residual, gate, *, tokens: int, stream=None):
        """``residual += float(fp16(x w^T)) * gate[row // tokens]`` in place
        (out-projection + gate_add_half_f32); ``residual`` fp32 ``[m, n]``,
        ``gate`` fp32 ``[images, n]``."""
        d = self._desc(x, w, residual, PROJ_GATE_ADD, tokens)
        d.gate = gate.data_ptr()
        d.gate_stride = gate.stride(0)
        return self._run(d, x, w, residual, stream)
