"""CPU oracle for the paged-attention hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the checker (or as the timed CPU baseline).  The b2pa
package never imports it.

It restates, without importing, three pieces of the reference
(jacobzhang22/efficient-inference-system):

* ``paged_attention_np`` -- the torch reference attention
  (src/kernels/reference_paged_attention.py:10-59), vectorised per
  (sequence, head) with numpy in float32;
* ``paged_attention_c`` -- the same loop nest in C (oracle/paged_oracle.c),
  threaded with OpenMP; this is also the CPU baseline bench.py times;
* ``OraclePool`` / ``oracle_append_batch`` -- the block pool allocator
  (LayerBlockPool, src/cache/paged_kv.py:9-93) and the batched append
  (PagedKVCacheState.append :102-120, BatchedPagedKVCache.append_batch
  :151-172) on numpy arrays.

Pinning: tests/test_oracle_golden.py checks all three against golden vectors
produced by running the reference itself (tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "liboracle.so"


# ------------------------------------------------------------------ attention
def visible_count(seq_len: int, cur_len: int, t: int) -> int:
    """Keys row t sees: tokens j < seq_len with j <= seq_len - cur_len + t
    (reference_paged_attention.py:36,40-42)."""
    return max(0, min(seq_len, seq_len - cur_len + t + 1))


def gather_tokens(pool: np.ndarray, block_ids, h: int, n: int) -> np.ndarray:
    """Rows 0..n-1 of head h through the block table (reference_paged_attention.py:44-47)."""
    bs = pool.shape[2]
    if n == 0:
        return np.zeros((0, pool.shape[3]), dtype=pool.dtype)
    nb = -(-n // bs)
    ids = np.asarray(block_ids[:nb], dtype=np.int64)
    return pool[ids, h].reshape(nb * bs, pool.shape[3])[:n]


def paged_attention_np(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, block_tables, seq_lens,
                       cur_lens) -> np.ndarray:
    """float32 restatement of paged_attention_reference.

    q: [B,H,T,D]; pools [NB,H,BS,D]; block_tables: list of block-id lists;
    seq_lens: lengths after the append; cur_lens: tokens added this step
    (None -> T for every row, an int -> the same for every row).
    """
    q = np.asarray(q, dtype=np.float32)
    k_pool = np.asarray(k_pool, dtype=np.float32)
    v_pool = np.asarray(v_pool, dtype=np.float32)
    B, H, T, D = q.shape
    if cur_lens is None:
        cur_lens = [T] * B
    elif isinstance(cur_lens, int):
        cur_lens = [cur_lens] * B
    scale = np.float32(1.0 / math.sqrt(D))
    out = np.zeros_like(q)
    for b in range(B):
        L = int(seq_lens[b])
        c = int(cur_lens[b])
        n_max = max(visible_count(L, c, t) for t in range(T)) if T else 0
        if n_max == 0:
            continue
        for h in range(H):
            K = gather_tokens(k_pool, block_tables[b], h, n_max)
            V = gather_tokens(v_pool, block_tables[b], h, n_max)
            s = (q[b, h] @ K.T) * scale  # [T, n_max]
            for t in range(T):
                n = visible_count(L, c, t)
                if n == 0:
                    continue
                row = s[t, :n]
                w = np.exp(row - row.max())
                w = w / w.sum()
                out[b, h, t] = w @ V[:n]
    return out


# ---------------------------------------------------------------- C oracle
def build_c_oracle(force: bool = False) -> Path:
    """Compiles oracle/paged_oracle.c into oracle/liboracle.so."""
    src = ORACLE_DIR / "paged_oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "liboracle.so"], check=True)
    return LIB_PATH


_clib = None


def _load_c():
    global _clib
    if _clib is None:
        build_c_oracle()
        lib = ctypes.CDLL(str(LIB_PATH))
        vp = ctypes.c_void_p
        lib.oracle_paged_attention_f32.restype = ctypes.c_int
        lib.oracle_paged_attention_f32.argtypes = [vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                   ctypes.c_int, vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int,
                                                   ctypes.c_float, ctypes.c_int]
        lib.oracle_max_threads.restype = ctypes.c_int
        _clib = lib
    return _clib


def c_max_threads() -> int:
    return int(_load_c().oracle_max_threads())


def paged_attention_c(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, block_tables, seq_lens, cur_lens,
                      nthreads: int = 0) -> np.ndarray:
    """Same contract as ``paged_attention_np``, computed by paged_oracle.c."""
    lib = _load_c()
    q = np.ascontiguousarray(q, dtype=np.float32)
    k_pool = np.ascontiguousarray(k_pool, dtype=np.float32)
    v_pool = np.ascontiguousarray(v_pool, dtype=np.float32)
    B, H, T, D = q.shape
    if cur_lens is None:
        cur_lens = [T] * B
    elif isinstance(cur_lens, int):
        cur_lens = [cur_lens] * B
    flat = np.concatenate([np.asarray(bt, dtype=np.int32) for bt in block_tables] + [np.zeros(1, np.int32)])
    offs = np.zeros(B, dtype=np.int64)
    acc = 0
    for b, bt in enumerate(block_tables):
        offs[b] = acc
        acc += len(bt)
    qs = np.array([s // 4 for s in q.strides], dtype=np.int64)
    sl = np.asarray(seq_lens, dtype=np.int32)
    cl = np.asarray(cur_lens, dtype=np.int32)
    out = np.empty((B, H, T, D), dtype=np.float32)
    rc = lib.oracle_paged_attention_f32(q.ctypes.data, qs.ctypes.data, k_pool.ctypes.data, v_pool.ctypes.data,
                                        k_pool.shape[0], H, k_pool.shape[2], D, flat.ctypes.data, offs.ctypes.data,
                                        sl.ctypes.data, cl.ctypes.data, out.ctypes.data, B, T,
                                        np.float32(1.0 / math.sqrt(D)), int(nthreads))
    if rc != 0:
        raise ValueError("oracle: block table references a block outside the pool")
    return out


# ------------------------------------------------------- allocator / append
class OraclePool:
    """Block pool bookkeeping + numpy storage (LayerBlockPool, paged_kv.py:9-93)."""

    def __init__(self, block_size: int, initial_blocks: int, growth_factor: float):
        self.block_size = block_size
        self.initial_blocks = initial_blocks
        self.growth_factor = growth_factor
        self.k = None
        self.v = None
        self.free: list[int] = []
        self.capacity = 0
        self.H = self.D = None
        self.dtype = None

    def ensure_initialized(self, H: int, D: int, dtype) -> None:
        if self.k is not None:
            return
        self.H, self.D, self.dtype = H, D, dtype
        self._grow(self.initial_blocks)

    def _grow(self, min_extra: int) -> None:
        # paged_kv.py:48-52: grow by max(min_extra, initial or ceil(cap*(g-1))), at least 1
        extra = self.initial_blocks if self.capacity == 0 else int(math.ceil(self.capacity * (self.growth_factor - 1.0)))
        grow_by = max(max(min_extra, extra), 1)
        new = np.zeros((grow_by, self.H, self.block_size, self.D), dtype=self.dtype)
        self.k = new.copy() if self.k is None else np.concatenate([self.k, new])
        self.v = new.copy() if self.v is None else np.concatenate([self.v, new])
        start = self.capacity
        self.capacity += grow_by
        self.free.extend(range(start, self.capacity))  # paged_kv.py:71-73

    def allocate(self) -> int:
        if not self.free:  # paged_kv.py:76-78
            self._grow(1)
        return self.free.pop()

    def release(self, block_id: int) -> None:
        if self.k is None:  # paged_kv.py:81-85
            return
        self.k[block_id] = 0
        self.v[block_id] = 0
        self.free.append(block_id)


class OracleState:
    def __init__(self, pool: OraclePool):
        self.pool = pool
        self.block_ids: list[int] = []
        self.seq_len = 0

    def append(self, k_new: np.ndarray, v_new: np.ndarray, length: int) -> None:
        """PagedKVCacheState.append (paged_kv.py:102-120); k_new: [H, T, D]."""
        if length <= 0:
            return
        H, _, D = k_new.shape
        self.pool.ensure_initialized(H, D, k_new.dtype)
        bs = self.pool.block_size
        offset = 0
        while offset < length:
            boff = self.seq_len % bs
            if boff == 0:
                self.block_ids.append(self.pool.allocate())
            blk = self.block_ids[-1]
            take = min(bs - boff, length - offset)
            self.pool.k[blk, :, boff:boff + take, :] = k_new[:, offset:offset + take, :]
            self.pool.v[blk, :, boff:boff + take, :] = v_new[:, offset:offset + take, :]
            self.seq_len += take
            offset += take

    def release(self) -> None:
        for blk in self.block_ids:
            self.pool.release(blk)
        self.block_ids.clear()
        self.seq_len = 0


def oracle_append_batch(states: list[OracleState], k_new: np.ndarray, v_new: np.ndarray, current_lengths) -> list[int]:
    """BatchedPagedKVCache.append_batch (paged_kv.py:151-172); k_new [B,H,T,D]."""
    B, _, T, _ = k_new.shape
    if current_lengths is None:
        lengths = [T] * B
    elif isinstance(current_lengths, int):
        lengths = [current_lengths] * B
    else:
        lengths = [int(x) for x in current_lengths]
    out = []
    for b, st in enumerate(states):
        st.append(k_new[b], v_new[b], max(min(lengths[b], T), 0))
        out.append(st.seq_len)
    return out


def page_table(states) -> np.ndarray:
    """-1 padded int32 [B, max_pages] (paged_kv.py:174-193)."""
    mp = max((len(s.block_ids) for s in states), default=0)
    t = np.full((len(states), mp), -1, dtype=np.int32)
    for r, s in enumerate(states):
        t[r, : len(s.block_ids)] = s.block_ids
    return t


# ------------------------------------------------------------ bf16 helpers
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Rounds float32 values to the nearest bfloat16 (ties to even), returned
    as float32 -- the values a bf16 tensor holds."""
    a = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (a >> 16) & 1
    r = ((a + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    nan = np.isnan(x)
    out = r.view(np.float32).copy()
    out[nan] = np.nan
    return out


def default_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
