"""KV append/scatter and block release on the GPU, bit-exact against the
reference's own pools (golden) and the CPU oracle's append."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import b2pa
from oracle import oracle as orc
from tests._helpers import load_golden

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy()
    return t.view(torch.int16).numpy()


def test_golden_alloc_sequence_bit_exact(cuda_device):
    g = load_golden("alloc_sequence")
    pool = b2pa.LayerBlockPool(int(g["block_size"]), int(g["initial_blocks"]), float(g["growth_factor"]))
    states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(3)]
    cache = b2pa.BatchedPagedKVCache(states, pool=pool)
    for i in range(int(g["n_steps"])):
        rel = int(g[f"step{i}_release"])
        if rel >= 0:
            states[rel].release()
        kind = str(g[f"step{i}_lens_kind"])
        lens = None if kind == "none" else (int(g[f"step{i}_lens"][0]) if kind == "int" else
                                            torch.tensor(g[f"step{i}_lens"]))
        k = torch.from_numpy(g[f"step{i}_k"]).to(cuda_device)
        v = torch.from_numpy(g[f"step{i}_v"]).to(cuda_device)
        ret = cache.append_batch(k, v, lens)
        assert ret.tolist() == g[f"step{i}_ret"].tolist()
        assert [b for s in states for b in s.block_ids] == g[f"step{i}_block_ids"].tolist()
        assert pool.free_block_ids == g[f"step{i}_free"].tolist()
    torch.cuda.synchronize()
    assert np.array_equal(_bits(pool.k_blocks), g["k_pool"].view(np.int32))
    assert np.array_equal(_bits(pool.v_blocks), g["v_pool"].view(np.int32))
    assert b2pa.read_status(cuda_device) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D,bs", [(64, 16), (128, 16), (16, 8), (256, 32), (32, 8)])
def test_random_appends_match_oracle_bit_exact(cuda_device, dtype, D, bs):
    rng = np.random.default_rng(D * 100 + bs)
    B, H = 7, 4
    pool = b2pa.LayerBlockPool(bs, 3, 2.0)
    states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(B)]
    cache = b2pa.BatchedPagedKVCache(states, pool=pool)
    mpool = orc.OraclePool(bs, 3, 2.0)
    mstates = [orc.OracleState(mpool) for _ in range(B)]
    np_dtype = {torch.float32: np.float32, torch.bfloat16: np.float32, torch.float16: np.float16}[dtype]
    for step, T in enumerate([1, 2 * bs + 3, 1, bs - 1, 1, bs + 1, 40]):
        lens = rng.integers(0, T + 1, size=B).tolist()
        lens[step % B] = T
        x = torch.randn(B, T, 2, H, D).to(dtype)  # strided views like the model's projections
        k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2)
        cache.append_batch(k.to(cuda_device), v.to(cuda_device), torch.tensor(lens))
        if dtype == torch.bfloat16:
            kn = k.view(torch.int16).numpy().astype(np.int16)
            vn = v.view(torch.int16).numpy().astype(np.int16)
        else:
            kn, vn = k.numpy().astype(np_dtype), v.numpy().astype(np_dtype)
        orc.oracle_append_batch(mstates, kn, vn, lens)
        assert [s.block_ids for s in states] == [s.block_ids for s in mstates]
        assert [s.seq_len for s in states] == [s.seq_len for s in mstates]
    if step >= 3:
        states[2].release()
        mstates[2].release()
    torch.cuda.synchronize()
    ref_k = mpool.k.view(np.int32) if dtype == torch.float32 else mpool.k.view(np.int16)
    ref_v = mpool.v.view(np.int32) if dtype == torch.float32 else mpool.v.view(np.int16)
    assert np.array_equal(_bits(pool.k_blocks), ref_k)
    assert np.array_equal(_bits(pool.v_blocks), ref_v)
    assert pool.free_block_ids == mpool.free
    assert b2pa.read_status(cuda_device) == 0


def test_release_zeroes_blocks(cuda_device):
    pool = b2pa.LayerBlockPool(16, 8, 2.0)
    states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(2)]
    cache = b2pa.BatchedPagedKVCache(states, pool=pool)
    k = torch.randn(2, 4, 50, 64, device=cuda_device)
    cache.append_batch(k, k.clone(), [50, 33])
    ids = list(states[0].block_ids)
    states[0].release()
    torch.cuda.synchronize()
    assert pool.k_blocks[ids].abs().sum().item() == 0 and pool.v_blocks[ids].abs().sum().item() == 0
    assert pool.k_blocks[states[1].block_ids].abs().sum().item() > 0
    assert pool.free_block_ids[-len(ids):] == ids


def test_bad_block_id_is_reported_not_faulted(cuda_device):
    """A page-table entry past the pool end is skipped and flagged in the
    status word; the kernel never touches memory outside the pool."""
    lib = b2pa.load_library()
    import ctypes

    from b2pa import _lib

    k_pool = torch.zeros(4, 2, 16, 64, device=cuda_device)
    v_pool = torch.zeros_like(k_pool)
    k_new = torch.randn(1, 2, 1, 64, device=cuda_device)
    page_table = torch.tensor([[7]], dtype=torch.int32, device=cuda_device)  # 7 >= 4 blocks
    zero = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    one = torch.ones(1, dtype=torch.int32, device=cuda_device)
    b2pa.clear_status(cuda_device)
    rc = lib.b2pa_kv_append(k_new.data_ptr(), _lib.strides4(k_new), k_new.data_ptr(), _lib.strides4(k_new),
                            k_pool.data_ptr(), v_pool.data_ptr(), _lib.strides4(k_pool), 4, page_table.data_ptr(), 1, 1,
                            zero.data_ptr(), one.data_ptr(), 1, 2, 1, 64, 16, 0,
                            _lib.status_buffer(cuda_device).data_ptr(), _lib.stream_handle(cuda_device))
    assert rc == 0
    assert b2pa.read_status(cuda_device) == -3
    b2pa.clear_status(cuda_device)
    assert k_pool.abs().sum().item() == 0
    del ctypes


def test_patch_table_writes_cells_and_reports_bad_index(cuda_device):
    """b2pa_patch_table writes each (index, value) pair; an index outside the
    table is skipped and flagged, the others still land."""
    from b2pa import _lib

    lib = b2pa.load_library()
    table = torch.full((4, 8), -1, dtype=torch.int32, device=cuda_device)
    pairs = torch.tensor([0, 5, 9, 7, 31, 2, 32, 99, -1, 4], dtype=torch.int32, device=cuda_device)
    b2pa.clear_status(cuda_device)
    rc = lib.b2pa_patch_table(table.data_ptr(), table.numel(), pairs.data_ptr(), 5,
                              _lib.status_buffer(cuda_device).data_ptr(), _lib.stream_handle(cuda_device))
    assert rc == 0
    want = np.full(32, -1, dtype=np.int32)
    want[0], want[9], want[31] = 5, 7, 2
    assert np.array_equal(table.cpu().numpy().reshape(-1), want)
    assert b2pa.read_status(cuda_device) == -1
    b2pa.clear_status(cuda_device)


def test_resident_table_patched_across_steps(cuda_device):
    """Many decode-style steps on one batch (the device table is patched in
    place, never re-uploaded whole): the device table equals the reference's
    page table after every step, including after a release and regrowth."""
    from b2pa.paged_kv import device_metadata

    pool = b2pa.LayerBlockPool(16, 64, 2.0)
    rng = np.random.default_rng(11)
    states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(5)]
    cache = b2pa.BatchedPagedKVCache(states, pool=pool)
    k = torch.randn(5, 2, 40, 32, device=cuda_device)
    cache.append_batch(k, k, [int(x) for x in rng.integers(1, 40, size=5)])
    for step in range(60):
        one = torch.randn(5, 2, 1, 32, device=cuda_device)
        cache.append_batch(one, one, 1)
        if step == 30:
            states[2].release()
        table, seq_lens, max_pages = device_metadata(cache, torch.device(cuda_device))
        want = cache.page_table_array()
        got = table.cpu().numpy()
        assert np.array_equal(got[:, :want.shape[1]], want)
        assert (got[:, want.shape[1]:] == -1).all()
        assert seq_lens.cpu().tolist() == [s.seq_len for s in states]
    assert b2pa.read_status(cuda_device) == 0
