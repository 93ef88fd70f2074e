"""A serving-style loop on the GPU: requests arrive, are prefilled in chunks,
decode, finish and release their blocks; every step wraps the live states in
a new BatchedPagedKVCache, as the reference's executors do
(src/serving/continuous_generate.py:15-33, src/inference/generate_with_cache.py:48-67).
Every attention output is checked against the CPU oracle and the pools stay
bit-exact with the oracle's append/release mirror throughout."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import b2pa
from oracle import oracle as orc
from tests._helpers import TOL

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_continuous_batching_loop(cuda_device, dtype):
    rng = np.random.default_rng(12)
    torch.manual_seed(12)
    H, D, bs, chunk = 4, 64, 16, 48
    pool = b2pa.LayerBlockPool(bs, 8, 2.0)
    mpool = orc.OraclePool(bs, 8, 2.0)
    live = []  # (state, mirror_state, prompt_left, decode_left)
    arrivals = [(int(rng.integers(5, 130)), int(rng.integers(1, 30))) for _ in range(14)]
    step = 0
    while arrivals or live:
        step += 1
        while arrivals and len(live) < 5:
            p, d = arrivals.pop(0)
            live.append([b2pa.PagedKVCacheState(pool=pool), orc.OracleState(mpool), p, d])
        prefill = [r for r in live if r[2] > 0]
        group = prefill if prefill and step % 2 else [r for r in live if r[2] == 0] or prefill
        if group is prefill:
            lens = [min(chunk, r[2]) for r in group]
            T = max(lens)
        else:
            lens = [1] * len(group)
            T = 1
        B = len(group)
        x = torch.randn(B, T, 3, H, D).to(dtype)
        k, v, q = (x[:, :, i].transpose(1, 2) for i in range(3))
        cache = b2pa.BatchedPagedKVCache([r[0] for r in group], pool=pool)
        cache.append_batch(k.to(cuda_device), v.to(cuda_device), torch.tensor(lens))
        kn = k.float().numpy() if dtype == torch.float32 else k.view(torch.int16).numpy()
        vn = v.float().numpy() if dtype == torch.float32 else v.view(torch.int16).numpy()
        orc.oracle_append_batch([r[1] for r in group], kn, vn, lens)
        cur = torch.tensor(lens, device=cuda_device) if step % 3 else lens
        out = b2pa.paged_attention("triton_paged", q.to(cuda_device), cache, cur)
        mk = mpool.k if dtype == torch.float32 else (mpool.k.astype(np.uint32) << 16).view(np.float32)
        mv = mpool.v if dtype == torch.float32 else (mpool.v.astype(np.uint32) << 16).view(np.float32)
        ref = orc.paged_attention_c(q.float().numpy(), mk, mv, [r[1].block_ids for r in group],
                                    [r[1].seq_len for r in group], lens)
        np.testing.assert_allclose(out.float().cpu().numpy(), ref, **TOL[dtype])
        for r, n in zip(group, lens):
            if r[2] > 0:
                r[2] -= n
            else:
                r[3] -= 1
        for r in [r for r in live if r[2] == 0 and r[3] <= 0]:
            r[0].release()
            r[1].release()
            live.remove(r)
        assert [s for s in pool.free_block_ids] == mpool.free
    torch.cuda.synchronize()
    kb = pool.k_blocks.cpu()
    kb = kb.view(torch.int32).numpy() if dtype == torch.float32 else kb.view(torch.int16).numpy()
    ref_k = mpool.k.view(np.int32) if dtype == torch.float32 else mpool.k.view(np.int16)
    assert np.array_equal(kb, ref_k)
    assert b2pa.read_status(cuda_device) == 0
