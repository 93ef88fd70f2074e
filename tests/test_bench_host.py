"""Host-side logic of bench.py, on the CPU: the token-balanced partition of
sequences over ranks and the parity check of the benchmarked launch (run
here on CPU tensors standing in for the device buffers)."""
from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import bench
from oracle import oracle as orc


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("scaling", ["weak", "strong"])
def test_partition_covers_the_draw_with_equal_counts_and_balanced_tokens(world, scaling):
    args = SimpleNamespace(seqs=512, scaling=scaling)
    draw = bench.all_lengths(512 * world if scaling == "weak" else 512)
    parts = bench.balanced_partition(draw, world)
    assert sorted(np.concatenate(parts).tolist()) == list(range(len(draw)))
    assert {len(p) for p in parts} == {len(draw) // world}
    sums = np.array([int(draw[p].sum()) for p in parts])
    assert sums.max() <= 1.005 * sums.mean()
    for r in range(world):
        assert np.array_equal(bench.my_sequences(args, r, world), draw[parts[r]])


def test_partition_uneven_counts():
    parts = bench.balanced_partition(np.array([5, 9, 1, 7, 3, 3, 8]), 3)
    assert sorted(len(p) for p in parts) == [2, 2, 3]


def _fake_workload(B=5, Hh=2, Dd=16, steps=3, seed=0):
    """A stand-in for bench.Workload on CPU tensors, with the same layout:
    the appends of ``steps`` steps already written, and ``out`` holding the
    oracle's attention for the last step."""
    rng = np.random.default_rng(seed)
    lens0 = rng.integers(20, 60, size=B).astype(np.int64)
    final = lens0 + steps
    pages = (final + bench.BS - 1) // bench.BS
    nb = int(pages.sum()) + 4
    perm = rng.permutation(nb).astype(np.int32)
    table = np.full((B, int(pages.max())), -1, dtype=np.int32)
    o = 0
    for b in range(B):
        table[b, :pages[b]] = perm[o:o + pages[b]]
        o += int(pages[b])
    g = torch.Generator().manual_seed(seed)
    k_pool = torch.randn(nb, Hh, bench.BS, Dd, generator=g).to(torch.bfloat16)
    v_pool = torch.randn(nb, Hh, bench.BS, Dd, generator=g).to(torch.bfloat16)
    x = torch.randn(B, 1, 3, Hh, Dd, generator=g).to(torch.bfloat16)
    k_new, v_new, q = (x[:, :, i].transpose(1, 2) for i in range(3))
    for b in range(B):
        for p in range(int(lens0[b]), int(final[b])):
            blk = int(table[b, p // bench.BS])
            k_pool[blk, :, p % bench.BS] = k_new[b, :, 0]
            v_pool[blk, :, p % bench.BS] = v_new[b, :, 0]
    tables = [[int(i) for i in table[b, :pages[b]]] for b in range(B)]
    ref = orc.paged_attention_c(q.float().numpy(), k_pool.float().numpy(), v_pool.float().numpy(), tables,
                                final.tolist(), [1] * B)
    out = torch.from_numpy(ref).to(torch.bfloat16)
    return SimpleNamespace(B=B, lens0=lens0, table=table, k_pool=k_pool, v_pool=v_pool, k_new=k_new,
                           v_new=v_new, q=q, out=out), steps - 1


@pytest.fixture
def small_dims(monkeypatch):
    monkeypatch.setattr(bench, "H", 2)
    monkeypatch.setattr(bench, "D", 16)


def test_launch_parity_passes_on_a_correct_launch(small_dims):
    wl, step = _fake_workload()
    p = bench.launch_parity(torch, wl, step)
    assert p["ok"] and p["outputs_ok"] and p["appended_rows_bit_exact"]
    assert p["seqs"] >= 3 and p["appended_rows_checked"] >= 3 * (step + 1)
    assert max(p["seq_lens"]) == int((wl.lens0 + step + 1).max())


def test_launch_parity_catches_a_wrong_output_and_a_wrong_row(small_dims):
    wl, step = _fake_workload()
    b = int(np.argmax(wl.lens0 + step + 1))  # always sampled
    wl.out[b, 1, 0, 3] += 0.5
    p = bench.launch_parity(torch, wl, step)
    assert not p["outputs_ok"] and not p["ok"] and p["appended_rows_bit_exact"]
    wl, step = _fake_workload()
    pos = int(wl.lens0[b])  # the first appended row of that sequence
    blk = int(wl.table[b, pos // bench.BS])
    wl.v_pool[blk, 0, pos % bench.BS, 0] = -wl.v_pool[blk, 0, pos % bench.BS, 0] + 1
    p = bench.launch_parity(torch, wl, step)
    assert not p["appended_rows_bit_exact"] and not p["ok"]
    assert math.isfinite(p["max_abs_err"])
