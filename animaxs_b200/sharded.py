"""Heads sharded across GPUs + one NCCL all-gather (the 16K-token DiT case).

Each rank of a ``torch.distributed`` group computes query heads
``head_range(rank, world, heads)`` of the attention for every query row (each
rank holds the full Q/K/V), and the library's own NCCL communicator
all-gathers the head slices so every rank ends with the complete output
(``animaxs_attn_forward_head_sharded``).  ``torch.distributed`` is used only
to share the 128-byte NCCL id; the collective itself runs inside the library.
The reference is a single-device app and has no counterpart.
"""

from __future__ import annotations

import ctypes

from . import _lib
from ._lib import AttentionValidationError, raise_for


def head_range(rank: int, world: int, heads: int) -> tuple[int, int]:
    """[begin, end) of the query heads rank ``rank`` computes."""
    if world <= 0 or heads % world:
        raise AttentionValidationError(_lib.ERR_INVALID_ARG,
                                       f"heads ({heads}) must be a multiple of world ({world})")
    if not 0 <= rank < world:
        raise AttentionValidationError(_lib.ERR_INVALID_ARG, f"rank {rank} outside [0, {world})")
    per = heads // world
    return rank * per, (rank + 1) * per


def share_unique_id(group=None, make_id=None) -> bytes:
    """Rank 0 creates the 128-byte id (``make_id`` or NCCL's), everyone gets it."""
    import torch.distributed as dist
    rank = dist.get_rank(group)
    payload = [None]
    if rank == 0:
        payload[0] = make_id() if make_id is not None else nccl_unique_id()
    dist.broadcast_object_list(payload, src=0, group=group)
    uid = payload[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise AttentionValidationError(_lib.ERR_INVALID_ARG, "NCCL unique id must be 128 bytes")
    return bytes(uid)


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    rc = _lib.lib().animaxs_comm_unique_id(buf)
    raise_for(rc, "ncclGetUniqueId failed (is libnccl.so.2 loadable?)")
    return buf.raw


class HeadShardedAttention:
    """Config-5 head-sharded attention over ``world`` GPUs (one rank per GPU)."""

    def __init__(self, executor, rank: int, world: int, unique_id: bytes):
        self.ex = executor
        self.rank, self.world = rank, world
        comm = ctypes.c_void_p()
        rc = _lib.lib().animaxs_comm_create(executor.handle, world, rank,
                                             ctypes.create_string_buffer(unique_id, 128),
                                             ctypes.byref(comm))
        raise_for(rc, executor.last_error())
        self._comm = comm

    def close(self):
        if getattr(self, "_comm", None):
            _lib.lib().animaxs_comm_destroy(self._comm)
            self._comm = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __call__(self, q, k, v, out=None, *, stream=None, **kw):
        """Same arguments as AttentionExecutor.attention; q/k/v/out are the FULL tensors."""
        import torch
        from .executor import _stream_handle
        if out is None:
            out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        desc = self.ex.strided_desc(q, k, v, out, **kw)
        if stream is None:
            stream = torch.cuda.current_stream(q.device)
        rc = _lib.lib().animaxs_attn_forward_head_sharded(
            self.ex.handle, self._comm, ctypes.byref(desc), q.data_ptr(), k.data_ptr(),
            v.data_ptr(), out.data_ptr(), _stream_handle(stream))
        raise_for(rc, self.ex.last_error())
        return out
