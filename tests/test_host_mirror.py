"""Host-side logic of the b2pa package, on CPU: block allocation order,
growth, release/reuse, page tables and error behaviour.  Pools live on the
``meta`` device, so no data moves and no kernel is needed.  The allocation
results are pinned against the reference's own (tests/golden/alloc_sequence)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import b2pa
from b2pa.paged_kv import plan_append
from tests._helpers import load_golden

META = torch.device("meta")


def _meta(*shape):
    return torch.empty(*shape, device=META)


def test_allocation_sequence_matches_reference():
    g = load_golden("alloc_sequence")
    pool = b2pa.LayerBlockPool(int(g["block_size"]), int(g["initial_blocks"]), float(g["growth_factor"]))
    states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(3)]
    cache = b2pa.BatchedPagedKVCache(states=states, pool=pool)
    H, D = int(g["H"]), int(g["D"])
    for i in range(int(g["n_steps"])):
        rel = int(g[f"step{i}_release"])
        if rel >= 0:
            states[rel].release()
        T = int(g[f"step{i}_T"])
        kind = str(g[f"step{i}_lens_kind"])
        lens = None if kind == "none" else (int(g[f"step{i}_lens"][0]) if kind == "int" else
                                            torch.tensor(g[f"step{i}_lens"]))
        ret = cache.append_batch(_meta(3, H, T, D), _meta(3, H, T, D), lens)
        assert ret.dtype == torch.long
        assert [s.seq_len for s in states] == g[f"step{i}_ret"].tolist()
        assert [b for s in states for b in s.block_ids] == g[f"step{i}_block_ids"].tolist()
        assert [len(s.block_ids) for s in states] == g[f"step{i}_block_counts"].tolist()
        assert pool.free_block_ids == g[f"step{i}_free"].tolist()
        assert pool.capacity_blocks == int(g[f"step{i}_capacity"])
        assert tuple(pool.k_blocks.shape) == (pool.capacity_blocks, H, int(g["block_size"]), D)


# The reference's own unit tests (tests/test_paged_kv.py:9-40), on meta pools.
def test_allocator_growth_and_reuse():
    pool = b2pa.LayerBlockPool(block_size=4, initial_blocks=1, growth_factor=2.0)
    state = b2pa.PagedKVCacheState(pool=pool)
    b2pa.BatchedPagedKVCache([state], pool=pool).append_batch(_meta(1, 2, 6, 8), _meta(1, 2, 6, 8), [6])
    assert pool.capacity_blocks >= 2
    allocated = list(state.block_ids)
    state.release()
    assert pool.allocate_block() in allocated


def test_block_boundary_append():
    pool = b2pa.LayerBlockPool(block_size=4, initial_blocks=2, growth_factor=2.0)
    state = b2pa.PagedKVCacheState(pool=pool)
    b2pa.BatchedPagedKVCache([state], pool=pool).append_batch(_meta(1, 2, 5, 8), _meta(1, 2, 5, 8), [5])
    assert state.seq_len == 5
    assert len(state.block_ids) == 2


def test_batched_page_table_handles_heterogeneous_lengths():
    pool = b2pa.LayerBlockPool(block_size=4, initial_blocks=4, growth_factor=2.0)
    states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(2)]
    batch = b2pa.BatchedPagedKVCache(states=states, pool=pool)
    batch.append_batch(_meta(2, 2, 4, 8), _meta(2, 2, 4, 8), current_lengths=torch.tensor([4, 2]))
    table = batch.page_table_array()
    assert table.shape == (2, 1)
    assert [s.seq_len for s in states] == [4, 2]


@pytest.mark.parametrize("bs", [8, 16, 32])
def test_block_boundaries_allocate_exactly(bs):
    pool = b2pa.LayerBlockPool(block_size=bs, initial_blocks=1, growth_factor=2.0)
    st = b2pa.PagedKVCacheState(pool=pool)
    cache = b2pa.BatchedPagedKVCache([st], pool=pool)
    total = 0
    for n in [1, bs - 1, 1, bs, bs + 1, 0, 3 * bs - 2]:
        cache.append_batch(_meta(1, 1, max(n, 1), 16), _meta(1, 1, max(n, 1), 16), [n])
        total += n
        assert st.seq_len == total
        assert len(st.block_ids) == -(-total // bs)
    assert len(set(st.block_ids)) == len(st.block_ids)


def test_page_table_padding_and_empty():
    pool = b2pa.LayerBlockPool(block_size=16, initial_blocks=4, growth_factor=2.0)
    states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(3)]
    cache = b2pa.BatchedPagedKVCache(states, pool=pool)
    assert cache.page_table_array().shape == (3, 0)
    cache.append_batch(_meta(3, 2, 40, 16), _meta(3, 2, 40, 16), [40, 0, 17])
    t = cache.page_table_array()
    assert t.dtype == np.int32 and t.shape == (3, 3)
    assert (t[1] == -1).all() and t[2, 2] == -1 and (t[0] >= 0).all()
    start = plan_append(cache, _meta(3, 2, 1, 16), [1, 1, 1])
    assert start == [40, 0, 17]


def test_states_must_share_the_pool():
    p1 = b2pa.LayerBlockPool(16, 4, 2.0)
    p2 = b2pa.LayerBlockPool(16, 4, 2.0)
    cache = b2pa.BatchedPagedKVCache([b2pa.PagedKVCacheState(pool=p1), b2pa.PagedKVCacheState(pool=p2)], pool=p1)
    with pytest.raises(ValueError):
        cache.append_batch(_meta(2, 1, 1, 16), _meta(2, 1, 1, 16), 1)


def test_no_cpu_path():
    pool = b2pa.LayerBlockPool(16, 4, 2.0)
    cache = b2pa.BatchedPagedKVCache([b2pa.PagedKVCacheState(pool=pool)], pool=pool)
    with pytest.raises(RuntimeError, match="CUDA"):
        cache.append_batch(torch.zeros(1, 2, 1, 16), torch.zeros(1, 2, 1, 16), 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        b2pa.paged_attention("b200_paged", torch.zeros(1, 2, 1, 16), cache, 1)


def test_backend_name_is_validated_like_the_reference():
    pool = b2pa.LayerBlockPool(16, 4, 2.0)
    cache = b2pa.BatchedPagedKVCache([b2pa.PagedKVCacheState(pool=pool)], pool=pool)
    with pytest.raises(ValueError, match="Unsupported paged attention backend"):
        b2pa.paged_attention("flash", torch.zeros(1, 2, 1, 16), cache, 1)
    assert "triton_paged" in b2pa.SUPPORTED_BACKENDS and "b200_paged" in b2pa.SUPPORTED_BACKENDS


def test_memory_accounting_matches_reference_formulas():
    pool = b2pa.LayerBlockPool(block_size=16, initial_blocks=4, growth_factor=2.0)
    st = b2pa.PagedKVCacheState(pool=pool)
    b2pa.BatchedPagedKVCache([st], pool=pool).append_batch(_meta(1, 8, 20, 64), _meta(1, 8, 20, 64), [20])
    es = 4
    assert pool.bytes_per_block() == 2 * 8 * 16 * 64 * es
    assert pool.reserved_bytes() == 4 * pool.bytes_per_block()
    assert st.live_bytes() == 20 * 8 * 64 * 2 * es
    assert st.reserved_bytes() == 2 * pool.bytes_per_block()
    assert st.fragmentation_bytes() == st.reserved_bytes() - st.live_bytes()


def test_incremental_block_table_matches_full_rebuild():
    """The cached host table (b2pa._metadata) patched row by row equals a full
    rebuild after appends across block boundaries, releases and re-appends."""
    from b2pa import _metadata

    rng = np.random.default_rng(3)
    pool = b2pa.LayerBlockPool(block_size=16, initial_blocks=4, growth_factor=2.0)
    states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(9)]
    cache = b2pa.BatchedPagedKVCache(states, pool=pool)
    ent = None
    for step in range(40):
        lens = rng.integers(0, 40, size=9).tolist()
        cache.append_batch(_meta(9, 1, 40, 16), _meta(9, 1, 40, 16), lens)
        if step % 7 == 3:
            states[step % 9].release()
        full = cache.page_table_array()
        if ent is None or full.shape[1] > ent.width:
            ent = _metadata._Entry(states, max(full.shape[1], 1) * 2)
        _metadata._refresh_rows(ent)
        w = full.shape[1]
        assert np.array_equal(ent.table[:, :w], full)
        assert (ent.table[:, w:] == -1).all()


def test_release_then_regrow_between_refreshes():
    """A release clears a row's list in place; if the row regrows before the
    next refresh (same list object, possibly longer than before), the rows
    marked by mark_shrunk_rows are rewritten whole, and the patch cells the
    refresh reports rebuild the same table."""
    from b2pa import _metadata

    rng = np.random.default_rng(5)
    pool = b2pa.LayerBlockPool(block_size=4, initial_blocks=8, growth_factor=2.0)
    states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(4)]
    cache = b2pa.BatchedPagedKVCache(states, pool=pool)
    cache.append_batch(_meta(4, 1, 9, 8), _meta(4, 1, 9, 8), [9, 5, 1, 7])
    ent = _metadata._Entry(states, 256)
    _metadata._refresh_rows(ent)
    shadow = ent.table.copy()
    for step in range(60):
        for r in rng.choice(4, size=int(rng.integers(0, 3)), replace=False):
            states[r].release()
        _metadata.mark_shrunk_rows(ent)  # what the append planner does before allocating
        lens = rng.integers(0, 9, size=4).tolist()
        cache.append_batch(_meta(4, 1, 9, 8), _meta(4, 1, 9, 8), lens)
        cells = []
        changed, max_pages = _metadata._refresh_rows(ent, None, states, cells)
        assert max_pages >= 0
        flat = shadow.reshape(-1)
        flat[np.asarray(cells[0::2], dtype=np.int64)] = cells[1::2]
        full = cache.page_table_array()
        w = full.shape[1]
        assert np.array_equal(ent.table[:, :w], full)
        assert np.array_equal(shadow, ent.table)


def test_deferred_append_is_flushed_before_pool_changes(monkeypatch):
    """Host ordering of the deferred (fused) decode append: a pending row copy
    is performed before anything else touches the pool -- the next
    append_batch, a release, pool growth -- and ``set_fused_append`` /
    ``flush_pending`` behave as documented.  The copy itself is recorded
    instead of launched (no GPU here)."""
    from b2pa import paged_kv as pk

    calls = []

    def fake_kv_append(cache, k, v, starts, lengths):
        calls.append((cache, list(starts), list(lengths)))
        return torch.zeros(len(cache.states), dtype=torch.int32, device=META)

    monkeypatch.setattr(pk, "_kv_append", fake_kv_append)
    prev = b2pa.set_fused_append(True)
    try:
        assert b2pa.set_fused_append(True) is True
        pool = b2pa.LayerBlockPool(16, 2, 2.0)
        states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(2)]
        cache = b2pa.BatchedPagedKVCache(states, pool=pool)
        # meta tensors never defer: there is nothing to launch
        cache.append_batch(_meta(2, 1, 1, 16), _meta(2, 1, 1, 16), 1)
        assert getattr(pool, "_b2pa_pending", None) is None
        b2pa.flush_pending(pool)  # nothing pending: no-op
        assert calls == []

        def pend(starts):
            out = torch.empty(2, dtype=torch.long, device=META)
            pool._b2pa_pending = pk._PendingAppend(cache, _meta(2, 1, 1, 16), _meta(2, 1, 1, 16), starts, [1, 1],
                                                   out)

        pend([5, 6])
        cache.append_batch(_meta(2, 1, 1, 16), _meta(2, 1, 1, 16), 1)  # flushes first
        assert calls == [(cache, [5, 6], [1, 1])] and pool._b2pa_pending is None
        pend([7, 8])
        states[0].release()  # flush before the blocks are zeroed and freed
        assert calls[-1] == (cache, [7, 8], [1, 1]) and pool._b2pa_pending is None
        pend([9, 9])
        pool._grow(1)  # flush before the pool tensors are replaced
        assert calls[-1] == (cache, [9, 9], [1, 1]) and pool._b2pa_pending is None
        assert len(calls) == 3
    finally:
        b2pa.set_fused_append(prev)
    assert b2pa.set_fused_append(prev) == prev


def test_install_into_reference_rebinds_and_restores(tmp_path, monkeypatch):
    """install_into_reference on a stand-in package laid out like the
    reference (src/kernels/paged_attention.py, src/model/attention.py binding
    paged_attention by name, src/cache/paged_kv.py): all three call sites are
    rebound, CPU tensors and "paged_reference" still take the reference's own
    functions, an unknown backend is refused like the reference does,
    ``fuse_append`` switches the deferred append on, and uninstall() restores
    every original and the previous switch."""
    import importlib
    from types import SimpleNamespace

    from b2pa import paged_kv as pk

    pkg = tmp_path / "fakeref"
    files = {
        "__init__.py": "",
        "kernels/__init__.py": "from .paged_attention import paged_attention\n",
        "kernels/paged_attention.py": ("CALLS = []\n"
                                       "def paged_attention(backend, q, kv_cache, current_lengths):\n"
                                       "    CALLS.append(backend)\n"
                                       "    return 'reference attention'\n"),
        "model/__init__.py": "",
        "model/attention.py": "from fakeref.kernels.paged_attention import paged_attention\n",
        "cache/__init__.py": "",
        "cache/paged_kv.py": ("class BatchedPagedKVCache:\n"
                              "    def append_batch(self, k_new, v_new, current_lengths=None):\n"
                              "        return 'reference append'\n"),
    }
    for name, text in files.items():
        (pkg / name).parent.mkdir(parents=True, exist_ok=True)
        (pkg / name).write_text(text)
    monkeypatch.syspath_prepend(str(tmp_path))
    km = importlib.import_module("fakeref.kernels.paged_attention")
    mm = importlib.import_module("fakeref.model.attention")
    cm = importlib.import_module("fakeref.cache.paged_kv")
    kpkg = importlib.import_module("fakeref.kernels")
    orig_pa, orig_append = km.paged_attention, cm.BatchedPagedKVCache.append_batch

    prev = b2pa.set_fused_append(False)
    try:
        handle = b2pa.install_into_reference("fakeref", fuse_append=True)
        try:
            assert km.paged_attention is mm.paged_attention is kpkg.paged_attention
            assert km.paged_attention is not orig_pa
            assert cm.BatchedPagedKVCache.append_batch is not orig_append
            assert pk._fused_append is True
            cpu_q = torch.zeros(1, 1, 1, 4)
            assert mm.paged_attention("triton_paged", cpu_q, None, 1) == "reference attention"
            assert mm.paged_attention("paged_reference", SimpleNamespace(is_cuda=True), None, 1) == \
                "reference attention"
            assert km.CALLS == ["triton_paged", "paged_reference"]
            with pytest.raises(ValueError, match="Unsupported"):
                mm.paged_attention("nope", SimpleNamespace(is_cuda=True), None, 1)
            assert cm.BatchedPagedKVCache().append_batch(cpu_q, cpu_q, 1) == "reference append"
        finally:
            handle.uninstall()
        assert km.paged_attention is orig_pa and mm.paged_attention is orig_pa and kpkg.paged_attention is orig_pa
        assert cm.BatchedPagedKVCache.append_batch is orig_append
        assert pk._fused_append is False
    finally:
        b2pa.set_fused_append(prev)
