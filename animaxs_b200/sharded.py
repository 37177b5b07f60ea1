"""Heads sharded across GPUs (the 16K-token DiT case): the rank's heads, then
either one NCCL all-gather (:class:`HeadShardedAttention`) or, fused, the
attention kernel storing every output tile into every rank's output over
NVLink (:class:`PeerShardedAttention`).

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


class _DeviceArray:
    """A CUDA array interface over memory the library owns (no copy)."""

    def __init__(self, ptr: int, shape, typestr: str = "<f2"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def exchange_handles(handle: bytes, group=None) -> bytes:
    """Every rank's 64-byte IPC handle, concatenated in rank order."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    got = [None] * world
    dist.all_gather_object(got, handle, group=group)
    if any(not isinstance(h, (bytes, bytearray)) or len(h) != 64 for h in got):
        raise AttentionValidationError(_lib.ERR_INVALID_ARG, "IPC handles must be 64 bytes")
    return b"".join(bytes(h) for h in got)


class PeerShardedAttention:
    """Config-5 head-sharded attention with the all-gather fused into the
    attention kernel: each rank's output buffer ([B, S, H, D] fp16, owned by
    the library, shared over CUDA IPC) receives every rank's heads directly
    from the kernels' epilogues (``animaxs_attn_forward_head_sharded_peer``).
    ``torch.distributed`` only carries the IPC handles at setup.  Every rank
    makes the same calls in the same order; ``output`` is valid until this
    rank's next call."""

    def __init__(self, executor, rank: int, world: int, out_shape, group=None, exchange=None,
                 layout: str = "token"):
        """``out_shape`` is ``[B, S, H, D]``; ``layout`` "token" stores it
        token-major (``[B, S, H, D]`` contiguous), "head" head-major
        (``[B, H, S, D]`` contiguous, ``output`` is the ``[B, S, H, D]`` view)."""
        import torch
        self.ex = executor
        self.rank, self.world = rank, world
        self.shape = tuple(int(x) for x in out_shape)
        if len(self.shape) != 4 or layout not in ("token", "head"):
            raise AttentionValidationError(_lib.ERR_INVALID_ARG, "out_shape [B, S, H, D]; layout token or head")
        nbytes = 2
        for x in self.shape:
            nbytes *= x
        lib = _lib.lib()
        grp = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        rc = lib.animaxs_peer_group_create(executor.handle, world, rank, nbytes, ctypes.byref(grp), handle)
        raise_for(rc, executor.last_error())
        self._group = grp
        try:
            allh = exchange(handle.raw) if exchange else exchange_handles(handle.raw, group)
            rc = lib.animaxs_peer_group_connect(grp, ctypes.create_string_buffer(allh, len(allh)))
            raise_for(rc, executor.last_error())
        except Exception:
            self.close()
            raise
        ptr = lib.animaxs_peer_group_output(grp)
        b, sq, h, d = self.shape
        dev = f"cuda:{executor.device}"
        if layout == "head":
            self.output = torch.as_tensor(_DeviceArray(ptr, (b, h, sq, d)), device=dev).permute(0, 2, 1, 3)
        else:
            self.output = torch.as_tensor(_DeviceArray(ptr, self.shape), device=dev)

    def close(self):
        """Free the group.  Every rank must be past its last call first --
        synchronised, then a barrier across the ranks (``dist.barrier()``) --
        because a slower peer may still be storing into this rank's buffer."""
        if getattr(self, "_group", None):
            self.output = None
            _lib.lib().animaxs_peer_group_destroy(self._group)
            self._group = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __call__(self, q, k, v, *, stream=None, **kw):
        """Same arguments as AttentionExecutor.attention (q/k/v are the FULL
        tensors); returns ``output``, which holds every rank's heads."""
        import torch
        from .executor import _stream_handle
        desc = self.ex.strided_desc(q, k, v, self.output, **kw)
        if stream is None:
            stream = torch.cuda.current_stream(q.device)
        rc = _lib.lib().animaxs_attn_forward_head_sharded_peer(
            self.ex.handle, self._group, ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(),
            self.output.data_ptr(), _stream_handle(stream))
        raise_for(rc, self.ex.last_error())
        return self.output
