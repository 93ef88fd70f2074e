"""Host-side logic of the multi-GPU bench path on CPU with the gloo backend
(world size 2): every sequence is owned by exactly one rank, weak scaling
gives each rank the same count, timings reduce to the max over ranks, and
the launch parity check reduces to the worst rank."""
from __future__ import annotations

import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        for scaling in ("strong", "weak"):
            args = SimpleNamespace(scaling=scaling, seqs=37)
            mine = bench.my_sequences(args, rank, world)
            got = [None] * world
            dist.all_gather_object(got, mine.tolist())
            if rank == 0:
                np.save(os.path.join(out_dir, f"{scaling}.npy"), np.array(got, dtype=object), allow_pickle=True)
        t = bench.max_over_ranks([1.0 + rank, 5.0 - rank], torch.device("cpu"), world)
        if rank == 0:
            np.save(os.path.join(out_dir, "max.npy"), np.array(t))
        # parity of the benchmarked launch: worst case over ranks (rank 1's rows differ)
        mine = {"seqs": 5, "max_abs_err": 0.01 * (rank + 1), "tolerance": "t", "outputs_ok": True,
                "appended_rows_checked": 10 + rank, "appended_rows_bit_exact": rank == 0, "ok": rank == 0}
        red = bench.reduce_parity(torch, mine, torch.device("cpu"), world)
        if rank == 0:
            np.save(os.path.join(out_dir, "parity.npy"), np.array([red], dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_partition_and_max_reduction(tmp_path):
    import bench

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    strong = np.load(tmp_path / "strong.npy", allow_pickle=True)
    full = bench.all_lengths(37).tolist()
    merged = sorted(x for part in strong for x in part)
    assert merged == sorted(full)                       # strong: one shared set, split
    assert abs(len(strong[0]) - len(strong[1])) <= 1
    weak = np.load(tmp_path / "weak.npy", allow_pickle=True)
    assert len(weak[0]) == len(weak[1]) == 37           # weak: 37 per rank
    assert sorted(x for p in weak for x in p) == sorted(bench.all_lengths(74).tolist())
    assert np.load(tmp_path / "max.npy").tolist() == [2.0, 5.0]
    red = np.load(tmp_path / "parity.npy", allow_pickle=True)[0]
    assert red["seqs"] == 10 and red["ranks"] == 2 and red["appended_rows_checked"] == 21
    assert abs(red["max_abs_err"] - 0.02) < 1e-12
    assert red["ok"] is False and red["appended_rows_bit_exact"] is False


def _failing_worker(rank: int, world: int, port: int, out_dir: str, mode: str) -> None:
    """Rank 1 leaves (``mode == "exit"``) or stalls past the process-group
    timeout (``"slow"``) instead of joining the timing reduction; rank 0 must
    get an error from that collective, not wait for ever."""
    import datetime
    import time

    import torch
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        if mode == "slow":
            time.sleep(8)
        os._exit(0)  # leaves between steps, with no collective in flight
    t0 = time.monotonic()
    try:
        bench.max_over_ranks([1.0], torch.device("cpu"), world)
        outcome = "returned"
    except Exception as e:  # the backend's error type differs between closed peers and timeouts
        outcome = "raised " + type(e).__name__
    with open(os.path.join(out_dir, f"rank0_{mode}.txt"), "w") as f:
        f.write(f"{outcome} {time.monotonic() - t0:.2f}")
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "slow"])
def test_lost_rank_ends_the_reduction_with_an_error(tmp_path, mode):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path), mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    outcome, secs = (tmp_path / f"rank0_{mode}.txt").read_text().rsplit(" ", 1)
    assert outcome.startswith("raised"), outcome
    assert float(secs) < 30
