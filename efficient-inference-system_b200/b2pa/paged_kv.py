"""Paged KV cache: per-layer block pool, per-request block tables, batched view.

Host-side mirror of the reference's ``src/cache/paged_kv.py``
(jacobzhang22/efficient-inference-system).  Class names, attributes, the
allocation order and the return values are the reference's, so code written
against ``LayerBlockPool`` / ``PagedKVCacheState`` / ``BatchedPagedKVCache``
runs unchanged.  What differs is where the bytes move:

* block allocation stays on the host, exactly as in the reference
  (LIFO free list, geometric growth by ``torch.cat``; paged_kv.py:44-85);
* the K/V copies of a whole ``append_batch`` call are one launch of the
  ``b2pa_kv_append`` scatter kernel instead of two slice copies per touched
  block per request (paged_kv.py:109-120, 165-171);
* releasing a request zeroes all of its blocks with one ``b2pa_zero_blocks``
  launch instead of two ``zero_()`` calls per block (paged_kv.py:80-85).

Pools live on a CUDA device.  Pools on the ``meta`` device are accepted for
host-only bookkeeping (allocation order, page tables) with no data movement;
CPU pools are rejected -- there is no CPU path in this package.
"""
from __future__ import annotations

import ctypes
import itertools
import math
import operator
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._metadata import block_table_and_lengths, note_released_rows
from ._staging import stage_int32


class LayerBlockPool:
    """Block pool of one layer: K and V tensors ``[blocks, H, block_size, D]``.

    Mirrors ``LayerBlockPool`` (src/cache/paged_kv.py:9-93).
    """

    def __init__(self, block_size: int, initial_blocks: int, growth_factor: float):
        self.block_size = block_size
        self.initial_blocks = initial_blocks
        self.growth_factor = growth_factor
        self.k_blocks: torch.Tensor | None = None
        self.v_blocks: torch.Tensor | None = None
        self.num_heads: int | None = None
        self.head_dim: int | None = None
        self.dtype: torch.dtype | None = None
        self.device: torch.device | None = None
        self.free_block_ids: list[int] = []
        self.capacity_blocks = 0
        self._b2pa_pending = None  # a deferred decode append (set_fused_append)

    def ensure_initialized(self, num_heads: int, head_dim: int, dtype: torch.dtype, device: torch.device) -> None:
        """Lazily allocates the pool on first use (paged_kv.py:28-42)."""
        if self.k_blocks is not None:
            return
        device = torch.device(device)
        if device.type not in ("cuda", "meta"):
            raise RuntimeError(f"b2pa pools live on CUDA devices (or 'meta' for bookkeeping), not {device}")
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = device
        self._grow(self.initial_blocks)

    def _grow(self, min_extra_blocks: int) -> None:
        """Geometric growth, same arithmetic as paged_kv.py:44-73."""
        if self.num_heads is None or self.head_dim is None or self.dtype is None or self.device is None:
            raise ValueError("Pool must be initialized before growth.")
        if getattr(self, "_b2pa_pending", None) is not None:
            flush_pending(self)  # the copy below must carry the pending row
        grow_by = max(
            min_extra_blocks,
            self.initial_blocks if self.capacity_blocks == 0
            else int(math.ceil(self.capacity_blocks * (self.growth_factor - 1.0))),
        )
        grow_by = max(grow_by, 1)
        new_k = torch.zeros(grow_by, self.num_heads, self.block_size, self.head_dim, dtype=self.dtype,
                            device=self.device)
        new_v = torch.zeros_like(new_k)
        if self.k_blocks is None:
            self.k_blocks = new_k
            self.v_blocks = new_v
        else:
            self.k_blocks = torch.cat([self.k_blocks, new_k], dim=0)
            self.v_blocks = torch.cat([self.v_blocks, new_v], dim=0)
        start = self.capacity_blocks
        self.capacity_blocks += grow_by
        self.free_block_ids.extend(range(start, self.capacity_blocks))

    def allocate_block(self) -> int:
        """LIFO pop, growing by at least one block when empty (paged_kv.py:75-78)."""
        if not self.free_block_ids:
            self._grow(1)
        return self.free_block_ids.pop()

    def release_block(self, block_id: int) -> None:
        """Zeroes one block and returns it to the free list (paged_kv.py:80-85)."""
        self.release_blocks([block_id])

    def release_blocks(self, block_ids: list[int]) -> None:
        """Zeroes ``block_ids`` in one kernel launch, then frees them in order."""
        if self.k_blocks is None or self.v_blocks is None:
            return
        if getattr(self, "_b2pa_pending", None) is not None:
            flush_pending(self)  # a pending row must not land in a released block
        if block_ids and self.k_blocks.device.type == "cuda":
            _zero_blocks(self, block_ids)
        self.free_block_ids.extend(block_ids)

    def bytes_per_block(self) -> int:
        if self.k_blocks is None:
            return 0
        return 2 * self.k_blocks[0].numel() * self.k_blocks.element_size()

    def reserved_bytes(self) -> int:
        return self.capacity_blocks * self.bytes_per_block()


@dataclass
class PagedKVCacheState:
    """Block table and length of one request in one layer (paged_kv.py:96-137)."""

    pool: LayerBlockPool
    block_ids: list[int] = field(default_factory=list)
    seq_len: int = 0

    def reserve(self, length: int) -> int:
        """Allocates the blocks ``length`` more tokens need and advances
        ``seq_len``; returns the position of the first new token."""
        return reserve_tokens(self, length)

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, length: int) -> None:
        """Appends the first ``length`` tokens of ``k_new[0]``/``v_new[0]``."""
        if length <= 0:
            return
        BatchedPagedKVCache([self], pool=self.pool).append_batch(k_new[:1], v_new[:1], [length])

    def release(self) -> None:
        self.pool.release_blocks(list(self.block_ids))
        self.block_ids.clear()
        self.seq_len = 0

    def live_bytes(self) -> int:
        if self.pool.k_blocks is None:
            return 0
        kb = self.pool.k_blocks
        return self.seq_len * kb.shape[1] * kb.shape[3] * 2 * kb.element_size()

    def reserved_bytes(self) -> int:
        return len(self.block_ids) * self.pool.bytes_per_block()

    def fragmentation_bytes(self) -> int:
        return self.reserved_bytes() - self.live_bytes()


def host_lengths(current_lengths, T: int, B: int) -> list[int]:
    """Per-request token counts as append_batch reads them (paged_kv.py:157-162)."""
    if current_lengths is None:
        return [T] * B
    if isinstance(current_lengths, int):
        return [current_lengths] * B
    if isinstance(current_lengths, torch.Tensor):
        return [int(x) for x in current_lengths.tolist()]
    return [int(x) for x in current_lengths]


class BatchedPagedKVCache:
    """The requests of one layer seen as a batch (paged_kv.py:140-206)."""

    def __init__(self, states: list[PagedKVCacheState], pool: LayerBlockPool | None = None):
        self.states = states
        if pool is not None:
            self.pool = pool
        else:
            non_null = next((state for state in states if state is not None), None)
            if non_null is None:
                raise ValueError("BatchedPagedKVCache needs a pool when all states are uninitialized.")
            self.pool = non_null.pool

    def plan_append(self, k_new: torch.Tensor, lengths: list[int]) -> list[int]:
        """Host half of ``append_batch``: initialises the pool and allocates
        blocks request by request; returns each request's start position."""
        return plan_append(self, k_new, lengths)

    def append_batch(self, k_new: torch.Tensor, v_new: torch.Tensor,
                     current_lengths: int | torch.Tensor | list[int] | None = None) -> torch.Tensor:
        """Writes each request's new tokens into its blocks; returns the new
        sequence lengths as int64 (paged_kv.py:151-172)."""
        return append_batch_into(self, k_new, v_new, current_lengths)

    def page_table_array(self) -> np.ndarray:
        """int32 ``[B, max_pages]`` block table, -1 padded (paged_kv.py:174-193)."""
        max_pages = max((len(s.block_ids) for s in self.states), default=0)
        table = np.full((len(self.states), max_pages), -1, dtype=np.int32)
        for row, s in enumerate(self.states):
            if s.block_ids:
                table[row, : len(s.block_ids)] = s.block_ids
        return table

    def page_table_tensor(self, device: torch.device | None = None) -> torch.Tensor:
        device = device or self.pool.device
        return torch.from_numpy(self.page_table_array()).to(device)

    def seq_lens_tensor(self, device: torch.device | None = None) -> torch.Tensor:
        device = device or self.pool.device
        return torch.tensor([s.seq_len for s in self.states], dtype=torch.int32, device=device)

    def live_bytes(self) -> int:
        return sum(s.live_bytes() for s in self.states)

    def reserved_bytes(self) -> int:
        return sum(s.reserved_bytes() for s in self.states)

    def fragmentation_bytes(self) -> int:
        return sum(s.fragmentation_bytes() for s in self.states)


# ------------------------------------------------- duck-typed host logic
# These functions read and write only the attributes the reference's own
# classes have (states, pool, block_ids, seq_len, allocate_block,
# ensure_initialized, block_size), so they serve both this module's classes
# and the reference's when the backend is installed into it.

def reserve_tokens(state, length: int) -> int:
    """Allocates blocks for ``length`` more tokens of ``state`` in the
    reference's order -- one block each time the write position reaches a
    block boundary (paged_kv.py:110-113) -- advances ``seq_len`` and returns
    the position of the first new token.  The pool must be initialised."""
    start = state.seq_len
    if length <= 0:
        return start
    bs = state.pool.block_size
    need = -(-(start + length) // bs) - (-(-start // bs))
    for _ in range(need):
        state.block_ids.append(state.pool.allocate_block())
    state.seq_len = start + length
    return start


_seq_len_of = operator.attrgetter("seq_len")
_pool_of = operator.attrgetter("pool")
_SMALL_BATCH = 64  # below this, plain Python loops beat numpy's per-call overhead


def plan_append(cache, k_new: torch.Tensor, lengths, as_array: bool = False):
    """Initialises the pool and allocates blocks request by request, in batch
    order (paged_kv.py:165-171); returns each request's start position (a
    list; for large batches with ``as_array`` the int64 array it was computed
    in, which the launch metadata takes without a conversion).

    For large batches the per-request arithmetic is vectorised and only
    requests whose write crosses into new blocks (one in ``block_size`` per
    decode step) run the allocation loop; small batches take a plain loop
    (numpy's per-call cost dominates there).  Either way requests are served
    in batch order, so the LIFO free list hands out the same ids as the
    reference's loop."""
    _, H, T, D = k_new.shape
    pool = cache.pool
    states = cache.states
    if len(states) <= _SMALL_BATCH:
        n = [T if x > T else (0 if x < 0 else int(x)) for x in lengths]
        if any(n):
            pool.ensure_initialized(H, D, k_new.dtype, k_new.device)
            if k_new.device.type == "cuda":
                note_released_rows(cache, k_new.device)
        bs = pool.block_size
        allocate = pool.allocate_block
        starts = []
        for state, nb in zip(states, n):
            if state.pool is not pool:
                raise ValueError("b2pa: all states of a BatchedPagedKVCache must share its pool")
            start = state.seq_len
            starts.append(start)
            if nb <= 0:
                continue
            # one block each time the write position reaches a block boundary
            # (paged_kv.py:110-113): blocks for positions start .. start+nb-1
            ids = state.block_ids
            for _ in range((start + nb + bs - 1) // bs - (start + bs - 1) // bs):
                ids.append(allocate())
            state.seq_len = start + nb
        return starts
    n = np.clip(np.asarray(lengths, dtype=np.int64), 0, T)
    if n.any():
        pool.ensure_initialized(H, D, k_new.dtype, k_new.device)
        if k_new.device.type == "cuda":
            note_released_rows(cache, k_new.device)
    if not all(map(operator.is_, map(_pool_of, states), itertools.repeat(pool))):
        raise ValueError("b2pa: all states of a BatchedPagedKVCache must share its pool")
    start = np.fromiter(map(_seq_len_of, states), dtype=np.int64, count=len(states))
    bs = pool.block_size
    # one block each time the write position reaches a block boundary
    # (paged_kv.py:110-113): blocks for positions start .. start+n-1
    need = np.where(n > 0, (start + n + bs - 1) // bs - (start + bs - 1) // bs, 0)
    allocate = pool.allocate_block
    for b in np.flatnonzero(need).tolist():
        ids = states[b].block_ids
        for _ in range(int(need[b])):
            ids.append(allocate())
    grown = np.flatnonzero(n)
    if len(grown) == len(states):
        for state, length in zip(states, (start + n).tolist()):
            state.seq_len = length
    else:
        ends = (start + n).tolist()
        for b in grown.tolist():
            states[b].seq_len = ends[b]
    return start if as_array else start.tolist()


def append_batch_into(cache, k_new: torch.Tensor, v_new: torch.Tensor, current_lengths=None) -> torch.Tensor:
    """``BatchedPagedKVCache.append_batch`` (paged_kv.py:151-172): host block
    allocation, then one scatter-kernel launch for every copied token."""
    step = getattr(cache.pool, "_b2pa_step", None)
    if step is not None:  # an open DecodeStep planned this append already
        return step.append(cache, k_new, v_new, current_lengths)
    B, H, T, D = k_new.shape
    if B != len(cache.states):
        raise ValueError(f"k_new has {B} rows for {len(cache.states)} states")
    if v_new.shape != k_new.shape or v_new.dtype != k_new.dtype:
        raise ValueError("k_new and v_new must have the same shape and dtype")
    lengths = host_lengths(current_lengths, T, B)
    if B <= _SMALL_BATCH:
        clamped = [T if x > T else (0 if x < 0 else x) for x in lengths]
        any_new = any(clamped)
    else:
        clamped = np.clip(np.asarray(lengths, dtype=np.int64), 0, T)
        any_new = bool(clamped.any())
    if any_new and k_new.device.type not in ("cuda", "meta"):
        raise RuntimeError("b2pa: k_new must be a CUDA tensor (this package has no CPU path)")
    pool = cache.pool
    if getattr(pool, "_b2pa_pending", None) is not None:
        flush_pending(pool)  # an earlier deferred append goes first
    starts = plan_append(cache, k_new, clamped, as_array=True)
    if any_new and k_new.device.type == "cuda":
        if _fused_append and k_new.stride(3) == 1 and v_new.stride(3) == 1:
            seq_out = torch.empty(B, dtype=torch.long, device=k_new.device)
            try:
                pool._b2pa_pending = _PendingAppend(cache, k_new, v_new, starts, clamped, seq_out)
                return seq_out
            except AttributeError:  # a pool that refuses new attributes: append now
                pass
        seq_lens = _kv_append(cache, k_new, v_new, starts, clamped)
        return seq_lens.to(torch.long)
    return torch.tensor([s.seq_len for s in cache.states], dtype=torch.long, device=k_new.device)


# ------------------------------------------------------ deferred (fused) append
# With the fused append on, append_batch allocates its blocks and advances
# seq_len on the host as usual, but leaves the K/V row copy pending on the
# pool; the paged_attention call that follows on the same batch object --
# the reference's order, src/model/attention.py:56-62 -- performs it in its
# own launches: inside the decode launch (b2pa_paged_decode_append) for a
# decode step, inside the page copy of the fp32 tensor-core prefill
# (b2pa_paged_prefill_append) for a prompt chunk.  Every other b2pa call that
# touches the pool first performs a pending copy with the ordinary append
# kernel.
_fused_append = False


def set_fused_append(enabled: bool) -> bool:
    """Turns the deferred, fused append on or off for the process; returns
    the previous setting.  Off by default.

    While it is on, the pool bytes of the last append_batch on a pool (and
    the int64 lengths it returned) are written by the next b2pa call on that
    pool: normally the paged_attention of the same batch.  Code
    that reads pool tensors directly in between, or releases or allocates
    blocks through objects other than this package's, must call
    ``flush_pending(pool)`` first."""
    global _fused_append
    prev = _fused_append
    _fused_append = bool(enabled)
    return prev


class _PendingAppend:
    __slots__ = ("cache", "k_new", "v_new", "starts", "lengths", "seq_out")

    def __init__(self, cache, k_new, v_new, starts, lengths, seq_out):
        self.cache = cache
        self.k_new = k_new
        self.v_new = v_new
        self.starts = starts
        self.lengths = lengths
        self.seq_out = seq_out


def take_pending(pool):
    """Removes and returns the pool's deferred append (None if none)."""
    pend = getattr(pool, "_b2pa_pending", None)
    if pend is not None:
        pool._b2pa_pending = None
    return pend


def flush_pending(pool) -> None:
    """Performs the pool's deferred decode append now, with the ordinary
    append kernel, and fills the lengths tensor append_batch returned."""
    pend = getattr(pool, "_b2pa_pending", None)
    if pend is not None and not isinstance(pend, _PendingAppend):
        raise RuntimeError("b2pa: the pool is inside an open DecodeStep whose attention has not run yet")
    pend = take_pending(pool)
    if pend is not None:
        seq_lens = _kv_append(pend.cache, pend.k_new, pend.v_new, pend.starts, pend.lengths)
        pend.seq_out.copy_(seq_lens)


# ----------------------------------------------------------------- launches
def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"b2pa: {what} must be a CUDA tensor (this package has no CPU path)")


def device_metadata(cache, device: torch.device, extra: list[list[int]] | None = None):
    """Block table and sequence lengths of ``cache`` (plus any ``extra`` int32
    rows) on the device: ``(page_table[B, width], seq_lens[B], extras...,
    max_pages)``.  The table is cached per batch and patched incrementally
    (see ``_metadata``).  Works on the reference's own cache objects as well as
    on this module's: only ``states[i].block_ids`` / ``seq_len`` are read."""
    return block_table_and_lengths(cache, device, extra)


def _kv_append(cache, k_new: torch.Tensor, v_new: torch.Tensor, starts: list[int], lengths: list[int]) -> None:
    _require_cuda(k_new, "k_new")
    _require_cuda(v_new, "v_new")
    pool = cache.pool
    kb, vb = pool.k_blocks, pool.v_blocks
    if kb.device != k_new.device:
        raise ValueError(f"pool on {kb.device} but k_new on {k_new.device}")
    B, H, T, D = k_new.shape
    dev = k_new.device
    page_table, seq_lens, start_t, len_t, max_pages = block_table_and_lengths(cache, dev, [starts, lengths],
                                                                               transient=True)
    lib = _lib.load()
    rc = lib.b2pa_kv_append(
        k_new.data_ptr(), _lib.strides4(k_new), v_new.data_ptr(), _lib.strides4(v_new),
        kb.data_ptr(), vb.data_ptr(), _lib.strides4(kb), kb.shape[0],
        page_table.data_ptr() if max_pages else None, page_table.stride(0), max_pages,
        start_t.data_ptr(), len_t.data_ptr(), B, H, T, D, pool.block_size, _lib.dtype_code(k_new.dtype),
        _lib.status_buffer(dev).data_ptr(), _lib.stream_handle(dev))
    _lib.check(rc, "b2pa_kv_append")
    return seq_lens


def _zero_blocks(pool: LayerBlockPool, block_ids: list[int]) -> None:
    kb, vb = pool.k_blocks, pool.v_blocks
    dev = kb.device
    ids = stage_int32(np.asarray(block_ids, dtype=np.int32), dev, transient=True)
    lib = _lib.load()
    rc = lib.b2pa_zero_blocks(kb.data_ptr(), vb.data_ptr(), _lib.strides4(kb), kb.shape[0], ids.data_ptr(),
                              len(block_ids), kb.shape[1], kb.shape[3], kb.shape[2], _lib.dtype_code(kb.dtype),
                              _lib.status_buffer(dev).data_ptr(), _lib.stream_handle(dev))
    _lib.check(rc, "b2pa_zero_blocks")
