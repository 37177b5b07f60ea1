"""ctypes binding of ``libanimaxs_attn.so`` (declared in ``include/animaxs_attn.h``).

Loading fails loudly when the library is missing: there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libanimaxs_attn.so")

OK = 0
ERR_INVALID_ARG = -1
ERR_UNSUPPORTED = -2
ERR_OOB = -3
ERR_CUDA = -4
ERR_TIMEOUT = -5
ERR_NO_DEVICE = -6
ERR_NCCL = -7
ERR_OVERFLOW = -8
ERR_SCRATCH_LIMIT = -9

QK_NONE, QK_RMS, QK_RMS_ROPE = 0, 1, 2
NUMERICS_LEGACY, NUMERICS_FP32, NUMERICS_BF16 = 0, 1, 2


class AttentionError(RuntimeError):
    """Base class; ``status`` holds the C status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class AttentionValidationError(AttentionError, ValueError):
    """Counterpart of the reference's ``AnimapkError.validation(String)``."""


class AttentionTimeoutError(AttentionError, TimeoutError):
    pass


class AttentionDeviceError(AttentionError):
    pass


def raise_for(status: int, message: str):
    if status == OK:
        return
    if status in (ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_OOB, ERR_OVERFLOW, ERR_SCRATCH_LIMIT):
        raise AttentionValidationError(status, message)
    if status == ERR_TIMEOUT:
        raise AttentionTimeoutError(status, message)
    raise AttentionDeviceError(status, message or f"status {status}")


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
        ("q_len", ctypes.c_int32), ("kv_len", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("q_tok_stride", ctypes.c_int64), ("q_head_stride", ctypes.c_int64), ("q_batch_stride", ctypes.c_int64),
        ("k_tok_stride", ctypes.c_int64), ("k_head_stride", ctypes.c_int64), ("k_batch_stride", ctypes.c_int64),
        ("v_tok_stride", ctypes.c_int64), ("v_head_stride", ctypes.c_int64), ("v_batch_stride", ctypes.c_int64),
        ("o_tok_stride", ctypes.c_int64), ("o_head_stride", ctypes.c_int64), ("o_batch_stride", ctypes.c_int64),
        ("causal", ctypes.c_int32), ("kv_valid_len", ctypes.c_int32),
        ("kv_valid_lens", ctypes.c_void_p),
        ("scale", ctypes.c_float), ("qk_norm", ctypes.c_int32), ("eps", ctypes.c_float),
        ("q_norm_weight", ctypes.c_void_p), ("k_norm_weight", ctypes.c_void_p),
        ("rope_table", ctypes.c_void_p), ("rope_rows", ctypes.c_int32), ("qk_norm_targets", ctypes.c_int32),
        ("q_bytes", ctypes.c_int64), ("k_bytes", ctypes.c_int64), ("v_bytes", ctypes.c_int64),
        ("o_bytes", ctypes.c_int64), ("numerics", ctypes.c_int32),
    ]


class ProjDesc(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
        ("x_stride", ctypes.c_int64), ("w_stride", ctypes.c_int64), ("out_stride", ctypes.c_int64),
        ("epilogue", ctypes.c_int32), ("tokens", ctypes.c_int32), ("qk_norm", ctypes.c_int32),
        ("q_cols", ctypes.c_int32), ("k_cols", ctypes.c_int32), ("rope_rows", ctypes.c_int32),
        ("q_norm_weight", ctypes.c_void_p), ("k_norm_weight", ctypes.c_void_p),
        ("rope_table", ctypes.c_void_p), ("eps", ctypes.c_float), ("w_storage", ctypes.c_int32),
        ("gate", ctypes.c_void_p), ("gate_stride", ctypes.c_int64),
        ("w_scale", ctypes.c_void_p), ("w_zero", ctypes.c_void_p), ("w_packed_stride", ctypes.c_int64),
    ]


PROJ_STORE, PROJ_QKV_NORM, PROJ_GATE_ADD = 0, 1, 2
WEIGHT_FP16, WEIGHT_W8, WEIGHT_W4 = 0, 1, 2

# name -> (restype, argtypes); every symbol the header declares.
ABI_VERSION = 3  # ANIMAXS_ATTN_ABI_VERSION in include/animaxs_attn.h

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_DESC = ctypes.POINTER(AttnDesc)
SIGNATURES = {
    "animaxs_attn_abi_version": (_I, []),
    "animaxs_attn_create": (_I, [_I, ctypes.POINTER(_P)]),
    "animaxs_attn_destroy": (_I, [_P]),
    "animaxs_attn_last_error": (ctypes.c_char_p, [_P]),
    "animaxs_attn_desc_init": (_I, [_DESC, _I, _I, _I, _I, _I, _I]),
    "animaxs_attn_validate": (_I, [_P, _DESC, _P, _P, _P, _P]),
    "animaxs_attn_forward": (_I, [_P, _DESC, _P, _P, _P, _P, _P]),
    "animaxs_attn_synchronize": (_I, [_P, _P]),
    "animaxs_attn_scratch_bytes": (_I, [_DESC, ctypes.POINTER(_I64)]),
    "animaxs_attn_query_tiles": (_I, [_P, ctypes.POINTER(_I64)]),
    "animaxs_attn_set_kernel_timing": (_I, [_P, _I]),
    "animaxs_attn_set_score_probe": (_I, [_P, _P]),
    "animaxs_attn_kernel_timing": (_I, [_P, ctypes.POINTER(_I64), ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_double)]),
    "animaxs_rms_rope_split_half": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I64, ctypes.c_float, _P]),
    "animaxs_rmsnorm_heads_half": (_I, [_P, _P, _P, _P, _I, _I, _I, _I64, ctypes.c_float, _P]),
    "animaxs_rope3d_table": (_I, [_I, _I, _I, ctypes.POINTER(ctypes.c_float)]),
    "animaxs_rope1d_table": (_I, [_I, _I, ctypes.c_double, ctypes.POINTER(ctypes.c_float)]),
    "animaxs_gqa_kv_head": (_I, [_I, _I, _I]),
    "animaxs_comm_unique_id": (_I, [_P]),
    "animaxs_comm_create": (_I, [_P, _I, _I, _P, ctypes.POINTER(_P)]),
    "animaxs_comm_destroy": (_I, [_P]),
    "animaxs_attn_forward_head_sharded": (_I, [_P, _P, _DESC, _P, _P, _P, _P, _P]),
    "animaxs_peer_group_create": (_I, [_P, _I, _I, _I64, ctypes.POINTER(_P), _P]),
    "animaxs_peer_group_connect": (_I, [_P, _P]),
    "animaxs_peer_group_output": (_P, [_P]),
    "animaxs_peer_group_destroy": (_I, [_P]),
    "animaxs_attn_forward_head_sharded_peer": (_I, [_P, _P, _DESC, _P, _P, _P, _P, _P]),
    "animaxs_attn_forward_noalloc": (_I, [_DESC, _P, _P, _P, _P, _P]),
    "animaxs_attn_noalloc_status": (_I, []),
    "animaxs_attn_selftest_wait_timeout": (_I, [_P, _I64, _P]),
    "animaxs_cross_kv_cache_bytes": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_I64)]),
    "animaxs_cross_kv_cache_create": (_I, [_P, _I, _I, _I, _I, _I, _P, _I64, ctypes.POINTER(_P)]),
    "animaxs_cross_kv_cache_destroy": (_I, [_P]),
    "animaxs_cross_kv_cache_fill": (_I, [_P, _I, _P, _I64, _I64, _P, _I64, _I64, _I, _P, ctypes.c_float, _P]),
    "animaxs_cross_kv_cache_project": (_I, [_P, _I, _P, _I64, _I, _P, _I64, _P, ctypes.c_float, _P]),
    "animaxs_cross_kv_cache_block": (_I, [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_I64),
                                          ctypes.POINTER(_I64), ctypes.POINTER(_I)]),
    "animaxs_cross_kv_cache_mark_ready": (_I, [_P, _I, _I]),
    "animaxs_cross_kv_cache_reset": (_I, [_P]),
    "animaxs_weight_streamer_create": (_I, [_P, _I64, _I, ctypes.POINTER(_P)]),
    "animaxs_weight_streamer_destroy": (_I, [_P]),
    "animaxs_weight_streamer_register_host": (_I, [_P, _P, _I64]),
    "animaxs_weight_streamer_load": (_I, [_P, _I, _P, _I64, _I64, _P]),
    "animaxs_weight_streamer_slot": (_P, [_P, _I]),
    "animaxs_weight_streamer_wait_loaded": (_I, [_P, _I, _P]),
    "animaxs_weight_streamer_mark_in_flight": (_I, [_P, _I, _P]),
    "animaxs_weight_streamer_complete": (_I, [_P, _I]),
    "animaxs_weight_streamer_state": (_I, [_P, _I, ctypes.POINTER(_I64), ctypes.POINTER(_I)]),
    "animaxs_proj_desc_init": (_I, [ctypes.POINTER(ProjDesc), _I, _I, _I, _I]),
    "animaxs_proj_validate": (_I, [_P, ctypes.POINTER(ProjDesc), _P, _P, _P]),
    "animaxs_proj_forward": (_I, [_P, ctypes.POINTER(ProjDesc), _P, _P, _P, _P]),
    "animaxs_dequant_to_half": (_I, [_P, _I, _P, _P, _P, _P, _I, _I, _I64, _I64, _P]),
}

_lib = None


def lib():
    """The loaded library (built in-tree by ``animaxs_b200.build``)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m animaxs_b200.build` "
                "(the attention path has no CPU fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.animaxs_attn_abi_version() != ABI_VERSION:
            raise ImportError(f"libanimaxs_attn.so ABI version mismatch (want {ABI_VERSION})")
        _lib = handle
    return _lib
