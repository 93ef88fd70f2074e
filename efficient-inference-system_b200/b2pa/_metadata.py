"""Device copies of a batch's block table and lengths, kept across calls.

The reference rebuilds the ``[B, max_pages]`` block table from Python lists
and copies it to the device on every attention call of every layer
(src/cache/paged_kv.py:174-193, src/kernels/paged_attention.py:25-26).  For
512 long sequences that is ~5 ms of host work per call.  Here one host table
per batch of request states is kept and patched in place: block lists only
grow (a block appended when the write position crosses a block boundary,
paged_kv.py:110-113) or are cleared on release (:122-126), so each call only
compares every row's list identity and length with the last snapshot and
copies the new tail of the rows that changed.  A release clears the list in
place, so a row released and regrown between two refreshes could keep both;
the append planner therefore marks shrunken rows (``note_released_rows``)
before it allocates.  The device table stays
resident: the cells that changed (one per sequence that crossed a block
boundary, in decode) go up as (index, value) pairs together with the lengths
(which change every step) and any per-call rows in one small pinned copy, and
b2pa_patch_table writes them in place; only a table that had to grow, or a
change of more than _MAX_PATCH_PAIRS cells, is uploaded whole.

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

from . import _lib
from ._staging import stage_int32

_MAX_ENTRIES = 64
# Up to this many changed cells the resident device table is patched in place
# (b2pa_patch_table); beyond it the whole table is uploaded again.
_MAX_PATCH_PAIRS = 1 << 16


class _Entry:
    __slots__ = ("states", "states_ref", "lists", "counts", "table", "dev_table", "width")

    def __init__(self, states, width: int):
        B = len(states)
        self.states = list(states)
        self.states_ref = states
        self.lists = [None] * B
        self.counts = [0] * B
        self.width = width
        self.table = np.full((B, width), -1, dtype=np.int32)
        self.dev_table: torch.Tensor | None = None


_entries: "OrderedDict[tuple, _Entry]" = OrderedDict()


def _refresh_rows(ent: _Entry, seq_out: np.ndarray | None = None, states=None,
                  cells: list | None = None) -> tuple[bool, int]:
    """Brings the host table up to date in one pass over the states; returns
    (any row changed, max block count) and fills ``seq_out`` with seq_len.
    A max block count of -1 asks the caller to rebuild the entry (a row
    outgrew the table, or ``states`` no longer holds the entry's states).
    With ``cells`` (a list), the flat index and new value of every table
    cell that changed are appended to it, interleaved."""
    changed = False
    table = ent.table
    counts = ent.counts
    lists = ent.lists
    mine = ent.states
    width = ent.width
    if states is not None and len(states) != len(mine):
        return True, -1
    max_pages = 0
    for r, s in enumerate(mine if states is None else states):
        if s is not mine[r]:
            return True, -1
        ids = s.block_ids
        n = len(ids)
        if n > max_pages:
            max_pages = n
        if seq_out is not None:
            seq_out[r] = s.seq_len
        old = counts[r]
        if n == old and ids is lists[r]:
            continue
        if n > width:
            return True, -1  # caller rebuilds a wider table
        if ids is lists[r] and n > old:
            table[r, old:n] = ids[old:n]
            if cells is not None:
                base = r * width
                for c in range(old, n):
                    cells.append(base + c)
                    cells.append(ids[c])
        else:
            table[r, :n] = ids
            if n < old:
                table[r, n:old] = -1
            if cells is not None:
                base = r * width
                for c in range(max(n, old)):
                    cells.append(base + c)
                    cells.append(ids[c] if c < n else -1)
        lists[r] = ids
        counts[r] = n
        changed = True
    return changed, max_pages


def _lookup(cache, device: torch.device, stream: int) -> _Entry | None:
    """The entry remembered on the batch object (the common case: the same
    batch object for append and attention), else the LRU by state identity."""
    ent = getattr(cache, "_b2pa_meta", None)
    if ent is not None and ent[0] == (device.index, stream) and ent[1].states_ref is cache.states:
        return ent[1]
    key = (device.index, stream, tuple(id(s) for s in cache.states))
    hit = _entries.get(key)
    if hit is not None:
        _entries.move_to_end(key)
    return hit


def mark_shrunk_rows(ent: _Entry) -> None:
    """Marks for a full rewrite every row whose block list is now shorter
    than the cached copy (a release: the reference clears the list in place,
    paged_kv.py:122-126, so once the row regrows, identity and length alone
    cannot show that its head changed)."""
    lists = ent.lists
    counts = ent.counts
    for r, s in enumerate(ent.states):
        if len(s.block_ids) < counts[r]:
            lists[r] = None


def note_released_rows(cache, device: torch.device) -> None:
    """Called by the append planner before it allocates blocks for ``cache``."""
    ent = _lookup(cache, device, _lib.stream_handle(device))
    if ent is not None:
        mark_shrunk_rows(ent)


def block_table_and_lengths(cache, device: torch.device, extra: list[list[int]] | None = None,
                            transient: bool = False):
    """Returns ``(page_table, seq_lens, *extras, max_pages)`` as int32 device
    tensors for the states of ``cache``.  ``page_table`` is ``[B, width]``
    with ``width >= max_pages`` (pass its row stride to the kernels).  With
    ``transient`` the lengths and extra rows live in a staging ring buffer:
    valid for work enqueued on the current stream right away (the launches
    of the calling function), not to be kept."""
    states = cache.states
    B = len(states)
    stream = _lib.stream_handle(device)
    rows = 1 + (len(extra) if extra else 0)
    small = np.empty(B * rows, dtype=np.int32)
    ent = _lookup(cache, device, stream)
    cells: list | None = [] if ent is not None and ent.dev_table is not None else None
    changed, max_pages = (True, -1) if ent is None else _refresh_rows(ent, small, states, cells)
    if max_pages < 0:
        max_pages = max((len(s.block_ids) for s in states), default=0)
        # headroom so that growing sequences do not force a rebuild (and a
        # whole-table upload) every few steps
        width = max(max_pages + max_pages // 8 + 8, 1)
        if ent is not None:
            width = max(width, ent.width * 2)
        ent = _Entry(states, width)
        key = (device.index, stream, tuple(id(s) for s in states))
        _entries[key] = ent
        while len(_entries) > _MAX_ENTRIES:
            _entries.popitem(last=False)
        cells = None
        changed, max_pages = _refresh_rows(ent, small)
    ent.states_ref = states
    try:
        cache._b2pa_meta = ((device.index, stream), ent)
    except AttributeError:  # batch objects that refuse new attributes use the LRU only
        pass
    if extra:
        for i, row in enumerate(extra):
            small[B * (i + 1): B * (i + 2)] = row  # a list, an array, or a scalar for equal values
    n_pairs = len(cells) // 2 if cells is not None else 0
    if ent.dev_table is not None and changed and 0 < n_pairs <= _MAX_PATCH_PAIRS:
        # few cells changed: send (index, value) pairs with the small rows and
        # patch the resident table in place
        packed = np.concatenate([small, np.asarray(cells, dtype=np.int32)])
        dev = stage_int32(packed, device, transient, stream)
        tail = dev[: B * rows]
        lib = _lib.load()
        _lib.check(lib.b2pa_patch_table(ent.dev_table.data_ptr(), ent.dev_table.numel(), dev[B * rows:].data_ptr(),
                                        n_pairs, _lib.status_buffer(device).data_ptr(), stream), "b2pa_patch_table")
    elif changed or ent.dev_table is None:
        packed = np.concatenate([ent.table.reshape(-1), small])
        dev = stage_int32(packed, device, False, stream)  # the resident table: kept
        ent.dev_table = dev[: B * ent.width].view(B, ent.width)
        tail = dev[B * ent.width:]
    else:
        tail = stage_int32(small, device, transient, stream)
    outs = [ent.dev_table]
    for i in range(rows):
        outs.append(tail[B * i: B * (i + 1)])
    outs.append(max_pages)
    return tuple(outs)


def clear() -> None:
    """Drops every cached table (tests use this to start cold)."""
    _entries.clear()
