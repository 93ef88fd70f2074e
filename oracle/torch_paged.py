"""Torch restatement of the reference's paged KV cache and torch attention --
TEST INFRASTRUCTURE ONLY (imported by tests/ and by oracle/model.py).

Runs on any torch device so end-to-end model tests can compare the b2pa
backend with the reference's semantics on the same GPU (same cuBLAS
projections, different attention path):

* ``TorchBlockPool`` / ``TorchCacheState`` / ``TorchBatchedCache`` restate
  LayerBlockPool, PagedKVCacheState and BatchedPagedKVCache
  (src/cache/paged_kv.py:9-206): LIFO allocation, geometric growth by
  torch.cat, per-block slice copies, release zeroing;
* ``paged_attention_torch`` restates paged_attention_reference
  (src/kernels/reference_paged_attention.py:10-59), vectorised per sequence:
  scores = q.K^T * scale, keys visible iff key <= seq_len - cur_len + t and
  key < seq_len, softmax, weighted sum; rows with no key are zero;
* ``paged_attention_token_loop`` restates the same function with the
  reference's own loop structure (one ``torch.dot`` per visible token and
  head), so that bench.py can time the reference's CPU path per
  (token, head) without the reference installed.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


class TorchBlockPool:
    def __init__(self, block_size: int, initial_blocks: int, growth_factor: float):
        self.block_size = block_size
        self.initial_blocks = initial_blocks
        self.growth_factor = growth_factor
        self.k_blocks = None
        self.v_blocks = None
        self.num_heads = self.head_dim = self.dtype = self.device = None
        self.free_block_ids: list[int] = []
        self.capacity_blocks = 0

    def ensure_initialized(self, num_heads, head_dim, dtype, device) -> None:
        if self.k_blocks is not None:
            return
        self.num_heads, self.head_dim, self.dtype, self.device = num_heads, head_dim, dtype, device
        self._grow(self.initial_blocks)

    def _grow(self, min_extra_blocks: int) -> None:  # paged_kv.py:44-73
        extra = (self.initial_blocks if self.capacity_blocks == 0
                 else int(math.ceil(self.capacity_blocks * (self.growth_factor - 1.0))))
        grow_by = max(max(min_extra_blocks, extra), 1)
        new_k = torch.zeros(grow_by, self.num_heads, self.block_size, self.head_dim, dtype=self.dtype,
                            device=self.device)
        new_v = torch.zeros_like(new_k)
        if self.k_blocks is None:
            self.k_blocks, self.v_blocks = new_k, new_v
        else:
            self.k_blocks = torch.cat([self.k_blocks, new_k], dim=0)
            self.v_blocks = torch.cat([self.v_blocks, new_v], dim=0)
        start = self.capacity_blocks
        self.capacity_blocks += grow_by
        self.free_block_ids.extend(range(start, self.capacity_blocks))

    def allocate_block(self) -> int:  # paged_kv.py:75-78
        if not self.free_block_ids:
            self._grow(1)
        return self.free_block_ids.pop()

    def release_block(self, block_id: int) -> None:  # paged_kv.py:80-85
        if self.k_blocks is None:
            return
        self.k_blocks[block_id].zero_()
        self.v_blocks[block_id].zero_()
        self.free_block_ids.append(block_id)


@dataclass
class TorchCacheState:
    pool: TorchBlockPool
    block_ids: list[int] = field(default_factory=list)
    seq_len: int = 0

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, length: int) -> None:  # paged_kv.py:102-120
        if length <= 0:
            return
        _, H, _, D = k_new.shape
        self.pool.ensure_initialized(H, D, k_new.dtype, k_new.device)
        bs = self.pool.block_size
        offset = 0
        while offset < length:
            boff = self.seq_len % bs
            if boff == 0:
                self.block_ids.append(self.pool.allocate_block())
            blk = self.block_ids[-1]
            take = min(bs - boff, length - offset)
            self.pool.k_blocks[blk, :, boff:boff + take, :] = k_new[0, :, offset:offset + take, :]
            self.pool.v_blocks[blk, :, boff:boff + take, :] = v_new[0, :, offset:offset + take, :]
            self.seq_len += take
            offset += take

    def release(self) -> None:
        for blk in self.block_ids:
            self.pool.release_block(blk)
        self.block_ids.clear()
        self.seq_len = 0


class TorchBatchedCache:
    def __init__(self, states, pool=None):
        self.states = states
        self.pool = pool if pool is not None else next(s for s in states if s is not None).pool

    def append_batch(self, k_new, v_new, current_lengths=None):  # paged_kv.py:151-172
        T = k_new.shape[2]
        if current_lengths is None:
            lengths = [T] * len(self.states)
        elif isinstance(current_lengths, int):
            lengths = [current_lengths] * len(self.states)
        else:
            lengths = [int(x) for x in current_lengths.tolist()]
        for b, st in enumerate(self.states):
            st.append(k_new[b:b + 1], v_new[b:b + 1], max(min(lengths[b], T), 0))
        return torch.tensor([s.seq_len for s in self.states], dtype=torch.long, device=k_new.device)


def paged_attention_torch(q: torch.Tensor, kv_cache, current_lengths) -> torch.Tensor:
    """reference_paged_attention.py:10-59, vectorised per sequence (same math,
    float32 accumulation in the dtype of q)."""
    B, H, T, D = q.shape
    if current_lengths is None:
        cur = [T] * B
    elif isinstance(current_lengths, int):
        cur = [current_lengths] * B
    else:
        cur = [int(x) for x in current_lengths.tolist()]
    out = torch.zeros_like(q)
    scale = 1.0 / math.sqrt(D)
    pool = kv_cache.pool
    bs = pool.block_size
    for b, st in enumerate(kv_cache.states):
        L = st.seq_len
        if L == 0:
            continue
        ids = torch.tensor(st.block_ids, dtype=torch.long, device=q.device)
        K = pool.k_blocks[ids].permute(1, 0, 2, 3).reshape(H, -1, D)[:, :L]   # [H, L, D]
        V = pool.v_blocks[ids].permute(1, 0, 2, 3).reshape(H, -1, D)[:, :L]
        s = torch.matmul(q[b], K.transpose(1, 2)) * scale                     # [H, T, L]
        past = L - cur[b]
        t_idx = torch.arange(T, device=q.device).view(T, 1)
        k_idx = torch.arange(L, device=q.device).view(1, L)
        vis = k_idx <= (past + t_idx)
        s = s.masked_fill(~vis, float("-inf"))
        any_vis = vis.any(dim=1)                                               # [T]
        w = torch.softmax(s, dim=-1)
        w = torch.where(any_vis.view(1, T, 1), w, torch.zeros_like(w))
        out[b] = torch.matmul(w, V)
    return out


def paged_attention_token_loop(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, block_ids: list[int],
                               seq_len: int, cur_len: int, heads=None) -> torch.Tensor:
    """The reference's CPU attention path with its cost structure kept: one
    sequence, a Python loop over (head, query row, visible token) with one
    pool row read for K and one for V and a ``torch.dot`` per token, then
    ``torch.stack`` / ``torch.softmax`` / weighted sum per row
    (reference_paged_attention.py:31-57).  ``paged_attention_torch`` above is
    the same math vectorised; this form exists to time what the reference's
    own loop costs per (token, head) on a CPU.  q: [H, T, D]; returns
    [len(heads), T, D] for the heads given (default all)."""
    H, T, D = q.shape
    bs = k_pool.shape[2]
    scale = 1.0 / math.sqrt(D)
    heads = range(H) if heads is None else heads
    out = torch.zeros(len(heads), T, D, dtype=q.dtype)
    first_query_pos = seq_len - cur_len
    for oh, h in enumerate(heads):
        for t in range(T):
            last = min(seq_len - 1, first_query_pos + t)
            if last < 0:
                continue
            scores, values = [], []
            qv = q[h, t]
            for j in range(last + 1):
                blk, off = block_ids[j // bs], j % bs
                scores.append(torch.dot(qv, k_pool[blk, h, off, :]) * scale)
                values.append(v_pool[blk, h, off, :])
            w = torch.softmax(torch.stack(scores), dim=0)
            out[oh, t] = torch.sum(w.unsqueeze(-1) * torch.stack(values, dim=0), dim=0)
    return out
