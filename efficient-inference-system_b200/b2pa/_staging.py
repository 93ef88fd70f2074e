"""Pinned host staging for the small int32 metadata uploads (block tables,
lengths, block-id lists).

The reference builds its page table with one ``torch.tensor(...).to(device)``
per request row (src/cache/paged_kv.py:186-192) -- a pageable, synchronous
copy each.  Here the whole metadata block goes up in one asynchronous copy
from a reusable pinned buffer.  Each pinned buffer carries a CUDA event so it
is only rewritten once the copy that last read it has finished.
"""
from __future__ import annotations

import threading

import numpy as np
import torch

_RING = 4


class _Slot:
    __slots__ = ("host", "event")

    def __init__(self, n: int):
        self.host = torch.empty(n, dtype=torch.int32, pin_memory=True)
        self.event: torch.cuda.Event | None = None


_lock = threading.Lock()
_rings: dict[int, list] = {}


def stage_int32(values: np.ndarray, device: torch.device) -> torch.Tensor:
    """Copies a 1-d int32 array to a fresh device tensor on the current stream."""
    n = int(values.size)
    out = torch.empty(n, dtype=torch.int32, device=device)
    if n == 0:
        return out
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _lock:
        ring = _rings.setdefault(idx, [0, [None] * _RING])
        pos = ring[0]
        ring[0] = (pos + 1) % _RING
        slot = ring[1][pos]
        if slot is None or slot.host.numel() < n:
            slot = _Slot(max(n, 4096) * 2)
            ring[1][pos] = slot
    if slot.event is not None:
        slot.event.synchronize()
    slot.host[:n].numpy()[:] = values.reshape(-1)
    out.copy_(slot.host[:n], non_blocking=True)
    ev = torch.cuda.Event()
    ev.record(torch.cuda.current_stream(device))
    slot.event = ev
    return out
