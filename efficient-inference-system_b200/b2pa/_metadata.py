"""Device copies of a batch's block table and lengths, kept across calls.

The reference rebuilds the ``[B, max_pages]`` block table from Python lists
and copies it to the device on every attention call of every layer
(src/cache/paged_kv.py:174-193, src/kernels/paged_attention.py:25-26).  For
512 long sequences that is ~5 ms of host work per call.  Here one host table
per batch of request states is kept and patched in place: block lists only
grow (a block appended when the write position crosses a block boundary,
paged_kv.py:110-113) or are cleared on release (:122-126), so each call only
compares every row's list identity and length with the last snapshot and
copies the new tail of the rows that changed.  The device table is uploaded
again only when a row changed; the lengths (which change every step) and any
per-call rows go up in one small pinned copy.

A batch is identified by the identity of its state objects and the current
stream (uploads are ordered on that stream only; the reference
builds a new BatchedPagedKVCache every step around the same states,
src/inference/generate_with_cache.py:48-67).  Entries hold strong references
to their states, so identities cannot be recycled while cached; the cache is a
small LRU.
"""
from __future__ import annotations

from collections import OrderedDict

import numpy as np
import torch

from ._staging import stage_int32

_MAX_ENTRIES = 64


class _Entry:
    __slots__ = ("states", "lists", "counts", "table", "dev_table", "width")

    def __init__(self, states, width: int):
        B = len(states)
        self.states = list(states)
        self.lists = [None] * B
        self.counts = np.zeros(B, dtype=np.int64)
        self.width = width
        self.table = np.full((B, width), -1, dtype=np.int32)
        self.dev_table: torch.Tensor | None = None


_entries: "OrderedDict[tuple, _Entry]" = OrderedDict()


def _refresh_rows(ent: _Entry) -> bool:
    """Brings the host table up to date; returns True if any row changed."""
    changed = False
    table = ent.table
    for r, s in enumerate(ent.states):
        ids = s.block_ids
        n = len(ids)
        old = int(ent.counts[r])
        if ids is ent.lists[r] and n == old:
            continue
        if ids is ent.lists[r] and n > old:
            table[r, old:n] = ids[old:n]
        else:
            table[r, :n] = ids
            if n < old:
                table[r, n:old] = -1
        ent.lists[r] = ids
        ent.counts[r] = n
        changed = True
    return changed


def block_table_and_lengths(cache, device: torch.device, extra: list[list[int]] | None = None):
    """Returns ``(page_table, seq_lens, *extras, max_pages)`` as int32 device
    tensors for the states of ``cache``.  ``page_table`` is ``[B, width]``
    with ``width >= max_pages`` (pass its row stride to the kernels)."""
    states = cache.states
    B = len(states)
    max_pages = max((len(s.block_ids) for s in states), default=0)
    key = (device.index, torch.cuda.current_stream(device).cuda_stream, tuple(id(s) for s in states))
    ent = _entries.get(key)
    if ent is None or max_pages > ent.width:
        width = max(max_pages, 1)
        if ent is not None:
            width = max(width, ent.width * 2)
        ent = _Entry(states, width)
        _entries[key] = ent
        while len(_entries) > _MAX_ENTRIES:
            _entries.popitem(last=False)
    else:
        _entries.move_to_end(key)
    dirty = _refresh_rows(ent) or ent.dev_table is None
    rows = 1 + (len(extra) if extra else 0)
    small = np.empty(B * rows, dtype=np.int32)
    small[:B] = [s.seq_len for s in states]
    if extra:
        for i, row in enumerate(extra):
            small[B * (i + 1): B * (i + 2)] = row
    if dirty:
        packed = np.concatenate([ent.table.reshape(-1), small])
        dev = stage_int32(packed, device)
        ent.dev_table = dev[: B * ent.width].view(B, ent.width)
        tail = dev[B * ent.width:]
    else:
        tail = stage_int32(small, device)
    outs = [ent.dev_table]
    for i in range(rows):
        outs.append(tail[B * i: B * (i + 1)])
    outs.append(max_pages)
    return tuple(outs)


def clear() -> None:
    """Drops every cached table (tests use this to start cold)."""
    _entries.clear()
