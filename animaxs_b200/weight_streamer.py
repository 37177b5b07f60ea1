"""Host mirror of the weight streamer (``animaxs_weight_streamer_*`` in
``include/animaxs_attn.h``): the reference's ``WeightStreamer``
(AnimaXS/Runtime/Metal/WeightStreamer.swift:84-213) -- bounded device memory
of 1 to 4 slots, each loaded with one execution range of a weight pack from
host memory, never overwritten while queued work still reads it.

The reference's names are kept (``capacity``, ``slot_count``, ``load``,
``buffer``, ``mark_in_flight``, ``complete``, ``loaded_logical_indexes``,
``in_flight_slot_set``).  Loads are asynchronous host-to-device copies on the
given stream; :meth:`wait_loaded` makes a consumer stream wait for a slot's
copy on the GPU, and a load into a slot marked in flight is ordered after the
marked work on the GPU (the reference refuses such a load on the host).
"""

from __future__ import annotations

import ctypes

from . import _lib
from .executor import AttentionExecutor, _stream_handle
from .sharded import _DeviceArray


class WeightStreamer:
    def __init__(self, executor: AttentionExecutor, capacity: int, slot_count: int = 1):
        self.ex = executor
        self._lib = executor._lib
        handle = ctypes.c_void_p()
        rc = self._lib.animaxs_weight_streamer_create(executor.handle, int(capacity), int(slot_count),
                                                      ctypes.byref(handle))
        executor._check(rc)
        self._h = handle
        self.capacity = int(capacity)
        self.slot_count = int(slot_count)
        self._pinned = []

    def register_host(self, array) -> None:
        """Pin a host range (a numpy array or a CPU torch tensor, e.g. a mapped
        pack) so that loads from it run as DMA; it must outlive the streamer."""
        ptr, nbytes = _host_ptr(array)
        self.ex._check(self._lib.animaxs_weight_streamer_register_host(self._h, ptr, nbytes))
        self._pinned.append(array)

    def load(self, src, *, slot: int = 0, logical_index: int = -1, nbytes: int | None = None,
             stream=None) -> None:
        """Copy host ``src`` (numpy array or CPU tensor, or (pointer, bytes))
        into ``slot`` on ``stream`` (default: the current torch stream)."""
        import torch
        ptr, size = _host_ptr(src)
        size = size if nbytes is None else int(nbytes)
        if stream is None:
            stream = torch.cuda.current_stream(self.ex.device)
        rc = self._lib.animaxs_weight_streamer_load(self._h, int(slot), ptr, size, int(logical_index),
                                                    _stream_handle(stream))
        self.ex._check(rc)

    def slot_ptr(self, slot: int) -> int:
        ptr = self._lib.animaxs_weight_streamer_slot(self._h, int(slot))
        if not ptr:
            raise _lib.AttentionValidationError(_lib.ERR_INVALID_ARG, f"weight slot {slot} out of range")
        return ptr

    def buffer(self, slot: int = 0, offset: int = 0, shape=None, dtype=None):
        """A torch view of ``slot`` (bytes by default) starting ``offset`` bytes in."""
        import torch
        dtype = torch.uint8 if dtype is None else dtype
        item = torch.empty((), dtype=dtype).element_size()
        shape = ((self.capacity - offset) // item,) if shape is None else tuple(shape)
        typestr = {torch.uint8: "|u1", torch.float16: "<f2", torch.float32: "<f4"}[dtype]
        arr = _DeviceArray(self.slot_ptr(slot) + int(offset), shape, typestr)
        return torch.as_tensor(arr, device=f"cuda:{self.ex.device}")

    def wait_loaded(self, slot: int, stream=None) -> None:
        import torch
        if stream is None:
            stream = torch.cuda.current_stream(self.ex.device)
        self.ex._check(self._lib.animaxs_weight_streamer_wait_loaded(self._h, int(slot), _stream_handle(stream)))

    def mark_in_flight(self, slot: int, stream=None) -> None:
        import torch
        if stream is None:
            stream = torch.cuda.current_stream(self.ex.device)
        self.ex._check(self._lib.animaxs_weight_streamer_mark_in_flight(self._h, int(slot),
                                                                        _stream_handle(stream)))

    def complete(self, slot: int) -> None:
        self.ex._check(self._lib.animaxs_weight_streamer_complete(self._h, int(slot)))

    def _state(self, slot):
        idx, fl = ctypes.c_int64(), ctypes.c_int()
        self.ex._check(self._lib.animaxs_weight_streamer_state(self._h, int(slot), ctypes.byref(idx),
                                                               ctypes.byref(fl)))
        return idx.value, bool(fl.value)

    @property
    def loaded_logical_indexes(self):
        return [None if i < 0 else i for i, _ in (self._state(s) for s in range(self.slot_count))]

    @property
    def in_flight_slot_set(self):
        return {s for s in range(self.slot_count) if self._state(s)[1]}

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.animaxs_weight_streamer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _host_ptr(src):
    if isinstance(src, tuple):
        return int(src[0]), int(src[1])
    if hasattr(src, "data_ptr"):
        if src.is_cuda:
            raise _lib.AttentionValidationError(_lib.ERR_INVALID_ARG, "weight loads come from host memory")
        return int(src.data_ptr()), int(src.numel() * src.element_size())
    return int(src.ctypes.data), int(src.nbytes)
