"""Host logic of b2pa.DecodeStep on the CPU: the lockstep allocation that
lets one block table serve every layer, on this package's pools (meta
device, bookkeeping only) and on the torch restatement of the reference's
pools."""
from __future__ import annotations

import pytest
import torch

import b2pa
from b2pa.step import reserve_lockstep
from oracle import torch_paged as tp


def _layers(pool_factory, n_layers=3, lens=(15, 16, 40, 1), init=4):
    pools = [pool_factory(16, init, 2.0) for _ in range(n_layers)]
    layers = []
    for pool in pools:
        pool.ensure_initialized(2, 8, torch.float32, torch.device("meta") if isinstance(pool, b2pa.LayerBlockPool)
                                else torch.device("cpu"))
        states = []
        for L in lens:
            st = (b2pa.PagedKVCacheState(pool=pool) if isinstance(pool, b2pa.LayerBlockPool)
                  else tp.TorchCacheState(pool=pool))
            for _ in range(-(-L // 16)):
                st.block_ids.append(pool.allocate_block())
            st.seq_len = L
            states.append(st)
        layers.append(states)
    return layers, pools


@pytest.mark.parametrize("factory", [b2pa.LayerBlockPool, tp.TorchBlockPool], ids=["b2pa", "reference_shaped"])
def test_lockstep_reservation_matches_per_layer_allocation(factory):
    layers, pools = _layers(factory)
    ref_layers, ref_pools = _layers(factory)
    for step in range(40):
        starts = reserve_lockstep(layers, pools)
        assert starts == [s.seq_len - 1 for s in layers[0]]
        # what each layer's own append would allocate, in batch order
        for states, pool in zip(ref_layers, ref_pools):
            for s in states:
                if s.seq_len % 16 == 0:
                    s.block_ids.append(pool.allocate_block())
                s.seq_len += 1
        for states, rstates in zip(layers, ref_layers):
            assert [s.block_ids for s in states] == [s.block_ids for s in rstates]
            assert [s.seq_len for s in states] == [s.seq_len for s in rstates]
        assert all(p.capacity_blocks == q.capacity_blocks for p, q in zip(pools, ref_pools))
    assert pools[0].capacity_blocks > 4  # the pools grew on the way


@pytest.mark.parametrize("factory", [b2pa.LayerBlockPool, tp.TorchBlockPool], ids=["b2pa", "reference_shaped"])
def test_lockstep_reservation_refuses_diverged_layers_without_changes(factory):
    layers, pools = _layers(factory)
    pools[2].free_block_ids.reverse()  # layer 2 would hand out other ids
    snapshot = [[(list(s.block_ids), s.seq_len) for s in states] for states in layers]
    with pytest.raises(RuntimeError, match="other block ids"):
        reserve_lockstep(layers, pools)
    assert snapshot == [[(list(s.block_ids), s.seq_len) for s in states] for states in layers]
    layers, pools = _layers(factory)
    layers[1][2].seq_len -= 1
    with pytest.raises(RuntimeError, match="not in\\s+lockstep"):
        reserve_lockstep(layers, pools)
