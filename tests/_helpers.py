"""Shared helpers for the test-suite: golden-fixture loading and synthetic
paged-cache construction.  Test infrastructure only."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"

# Tolerances from the task statement: fp32 rtol 1e-4 / atol 1e-5, bf16 2e-2.
TOL = {
    torch.float32: dict(rtol=1e-4, atol=1e-5),
    torch.bfloat16: dict(rtol=2e-2, atol=2e-2),
    torch.float16: dict(rtol=2e-2, atol=2e-2),
}


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def split_tables(flat: np.ndarray, counts: np.ndarray) -> list[list[int]]:
    out, o = [], 0
    for c in counts.tolist():
        out.append([int(x) for x in flat[o:o + c]])
        o += c
    return out


def golden_tensor(arr: np.ndarray, dtype_name: str) -> torch.Tensor:
    """Golden arrays: float32 as stored; bf16 stored as raw uint16 bits."""
    if dtype_name == "bfloat16":
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(arr))


def to_f32_numpy(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def random_tables(rng: np.random.Generator, lengths, num_blocks: int, block_size: int) -> list[list[int]]:
    """Non-overlapping random block tables drawn from a permutation of the pool."""
    pages = [-(-int(L) // block_size) for L in lengths]
    perm = rng.permutation(num_blocks)
    assert sum(pages) <= num_blocks
    out, o = [], 0
    for p in pages:
        out.append([int(x) for x in perm[o:o + p]])
        o += p
    return out


def build_cache(b2pa, k_pool: torch.Tensor, v_pool: torch.Tensor, tables, seq_lens, block_size: int):
    """A b2pa BatchedPagedKVCache over existing pool tensors and tables."""
    pool = b2pa.LayerBlockPool(block_size=block_size, initial_blocks=k_pool.shape[0], growth_factor=2.0)
    pool.k_blocks, pool.v_blocks = k_pool, v_pool
    pool.num_heads, pool.head_dim = k_pool.shape[1], k_pool.shape[3]
    pool.dtype, pool.device = k_pool.dtype, k_pool.device
    pool.capacity_blocks = k_pool.shape[0]
    used = {b for t in tables for b in t}
    pool.free_block_ids = [b for b in range(k_pool.shape[0]) if b not in used]
    states = [b2pa.PagedKVCacheState(pool=pool, block_ids=list(t), seq_len=int(L)) for t, L in zip(tables, seq_lens)]
    return b2pa.BatchedPagedKVCache(states=states, pool=pool)


def strided_q(B: int, H: int, T: int, D: int, dtype, device, gen=None) -> torch.Tensor:
    """q as the model produces it: a [B,H,T,D] view of a [B,T,H*D] projection
    (src/model/attention.py:25-29)."""
    x = torch.randn(B, T, H * D, generator=gen, device="cpu").to(dtype).to(device)
    return x.view(B, T, H, D).transpose(1, 2)
