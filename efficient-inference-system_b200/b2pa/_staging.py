"""Pinned host staging for the small int32 metadata uploads (block tables,
lengths, block-id lists).

The reference builds its page table with one ``torch.tensor(...).to(device)``
per request row (src/cache/paged_kv.py:186-192) -- a pageable, synchronous
copy each.  Here the whole metadata block goes up in one asynchronous copy
from a reusable pinned buffer.  Each pinned buffer carries a CUDA event so it
is only rewritten once the copy that last read it has finished.

Two kinds of upload:

* ``stage_int32(values, device)`` returns a fresh device tensor the caller
  may keep (the resident block table is one);
* ``stage_int32(values, device, transient=True)`` returns a view of a
  device buffer that belongs to a small per-stream ring: valid for work
  enqueued on the same stream before the ring comes round again (the next
  few uploads), which is how the kernel launches of one call use it.  It
  spares a device allocation per call.

The copies and events go straight to the CUDA runtime that torch itself
loaded (the per-call host cost matters: a decode step of a small model
makes two uploads per layer).
"""
from __future__ import annotations

import ctypes
import os
import threading

import numpy as np
import torch

_RING = 4
_H2D = 1  # cudaMemcpyHostToDevice
_EVENT_DISABLE_TIMING = 2

_rt = None


def _cudart():
    """The CUDA runtime library torch uses (same process-wide instance)."""
    global _rt
    if _rt is None:
        base = os.path.dirname(torch.__file__)
        names = [os.path.join(base, "..", "nvidia", "cuda_runtime", "lib", "libcudart.so.12"), "libcudart.so.12"]
        last = None
        for name in names:
            try:
                lib = ctypes.CDLL(name)
                break
            except OSError as e:  # try the next location
                last = e
        else:
            raise RuntimeError(f"b2pa: cannot load the CUDA runtime library: {last}")
        lib.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
        lib.cudaMemcpyAsync.restype = ctypes.c_int
        lib.cudaEventCreateWithFlags.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_uint]
        lib.cudaEventCreateWithFlags.restype = ctypes.c_int
        lib.cudaEventRecord.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.cudaEventRecord.restype = ctypes.c_int
        lib.cudaEventSynchronize.argtypes = [ctypes.c_void_p]
        lib.cudaEventSynchronize.restype = ctypes.c_int
        lib.cudaEventDestroy.argtypes = [ctypes.c_void_p]
        lib.cudaEventDestroy.restype = ctypes.c_int
        _rt = lib
    return _rt


def _rt_check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"b2pa: {what} failed with CUDA error {rc}")


class _Slot:
    __slots__ = ("host", "host_np", "dev", "event", "recorded")

    def __init__(self, n: int, device: torch.device, with_device: bool):
        self.host = torch.empty(n, dtype=torch.int32, pin_memory=True)
        self.host_np = self.host.numpy()
        self.dev = torch.empty(n, dtype=torch.int32, device=device) if with_device else None
        ev = ctypes.c_void_p()
        with torch.cuda.device(device):
            _rt_check(_cudart().cudaEventCreateWithFlags(ctypes.byref(ev), _EVENT_DISABLE_TIMING), "cudaEventCreate")
        self.event = ev
        self.recorded = False


_lock = threading.Lock()
_rings: dict[tuple, list] = {}


def _next_slot(key, n: int, device: torch.device, transient: bool) -> _Slot:
    with _lock:
        ring = _rings.setdefault(key, [0, [None] * _RING])
        pos = ring[0]
        ring[0] = (pos + 1) % _RING
        slot = ring[1][pos]
        if slot is None or slot.host.numel() < n:
            if slot is not None and slot.recorded:
                _rt_check(_cudart().cudaEventSynchronize(slot.event), "cudaEventSynchronize")
            slot = _Slot(max(n, 4096) * 2, device, transient)
            ring[1][pos] = slot
    return slot


def stage_int32(values: np.ndarray, device: torch.device, transient: bool = False,
                stream: int | None = None) -> torch.Tensor:
    """Copies a 1-d int32 array to the device on the current stream (or the
    raw ``stream`` handle given): a fresh tensor, or with ``transient`` a
    view of a per-stream ring buffer (see the module docstring)."""
    n = int(values.size)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if stream is None:
        stream = torch._C._cuda_getCurrentRawStream(idx)
    if n == 0:
        return torch.empty(0, dtype=torch.int32, device=device)
    dev_t = torch.device("cuda", idx)
    slot = _next_slot((idx, stream, transient), n, dev_t, transient)
    rt = _cudart()
    if slot.recorded:
        _rt_check(rt.cudaEventSynchronize(slot.event), "cudaEventSynchronize")
    slot.host_np[:n] = values.reshape(-1)
    out = slot.dev if transient else torch.empty(n, dtype=torch.int32, device=dev_t)
    _rt_check(rt.cudaMemcpyAsync(out.data_ptr(), slot.host.data_ptr(), 4 * n, _H2D, stream), "cudaMemcpyAsync")
    _rt_check(rt.cudaEventRecord(slot.event, stream), "cudaEventRecord")
    slot.recorded = True
    return out[:n] if transient else out
