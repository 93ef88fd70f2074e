"""b2pa.serving on the CPU: one rank reproduces the reference's continuous
scheduler (golden trace of the reference run with deterministic fake
executors); the router spreads requests by outstanding tokens; two gloo
ranks serve the config[3] trace with every request served by exactly one
rank and every rank holding every request's token stream."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch.multiprocessing as mp

import b2pa
from oracle import serving as osv
from tests._helpers import load_golden


def _trace():
    return osv.generate_requests(200, 52.0, 5000, osv.CONFIG3_PROFILES, seed=42)


def _expected_stream(r) -> list[int]:
    """The fake executors emit request_id % 97 when the prompt completes and
    request_id % 89 at every decode step."""
    return [r.request_id % 97] + [r.request_id % 89] * (r.max_new_tokens - 1)


def test_one_rank_reproduces_the_reference_scheduler():
    g = load_golden("serving_config3")
    res = b2pa.serve(_trace(), osv.fake_prefill_executor, osv.fake_decode_executor, max_batch_size=8,
                     prefill_chunk_size=256, max_tokens_per_iteration=1536)
    ev = res.events
    assert [e["phase"] for e in ev] == g["ev_phase"].tolist()
    assert [len(e["request_ids"]) for e in ev] == g["ev_batch_size"].tolist()
    assert [e["tokens_scheduled"] for e in ev] == g["ev_tokens"].tolist()
    np.testing.assert_allclose([e["dispatch_time_ms"] for e in ev], g["ev_dispatch_ms"], rtol=1e-12, atol=1e-9)
    done = res.completed
    assert [r.request_id for r in done] == list(range(200))
    np.testing.assert_allclose([r.first_token_time_ms for r in done], g["first_token_ms"], rtol=1e-12, atol=1e-9)
    np.testing.assert_allclose([r.finish_time_ms for r in done], g["finish_ms"], rtol=1e-12, atol=1e-9)
    # the restated scheduler the GPU tests use takes the same decisions
    _, ref_events = osv.ContinuousScheduler(8, 256, 1536).run(_trace(), osv.fake_prefill_executor,
                                                              osv.fake_decode_executor)
    assert [(e["phase"], e["request_ids"]) for e in ev] == [(p, ids) for p, ids, *_ in ref_events]
    assert all(res.token_streams[r.request_id] == _expected_stream(r) for r in done)


def test_router_least_outstanding_tokens():
    router = b2pa.LeastOutstandingTokensRouter(3)
    reqs = osv.generate_requests(6, 1000.0, 100, [osv.WorkloadProfile("w", 10, 10, 5, 5, 1.0)], seed=0)
    assert [router.route(r) for r in reqs[:3]] == [0, 1, 2]      # ties to the lowest rank
    router.sync([30, 0, 15])
    assert router.route(reqs[3]) == 1 and router.outstanding.tolist() == [30, 15, 15]
    assert router.route(reqs[4]) == 1                             # 15 == 15: the lower rank
    assert router.route(reqs[5]) == 2
    r = reqs[0]
    r.prompt_tokens_processed, r.generated_token_ids = 4, [1, 2]
    assert b2pa.serving.outstanding_tokens(r) == 6 + 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        res = b2pa.serve(_trace(), osv.fake_prefill_executor, osv.fake_decode_executor, max_batch_size=8,
                         prefill_chunk_size=256, max_tokens_per_iteration=1536, device=torch.device("cpu"))
        times = b2pa.gather_request_times(res.completed)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"),
                np.array([{"mine": [r.request_id for r in res.completed], "streams": res.token_streams,
                           "owner": res.owner, "times": times, "iterations": res.iterations,
                           "makespan": res.makespan_ms,
                           "outstanding_left": sum(b2pa.serving.outstanding_tokens(r) for r in res.completed)}],
                         dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_serve_the_trace(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    outs = [np.load(tmp_path / f"rank{r}.npy", allow_pickle=True)[0] for r in range(world)]
    reqs = {r.request_id: r for r in _trace()}
    mine = [set(o["mine"]) for o in outs]
    assert mine[0].isdisjoint(mine[1]) and (mine[0] | mine[1]) == set(reqs)   # each request on one rank
    assert outs[0]["owner"] == outs[1]["owner"]                               # same routing everywhere
    assert all(outs[0]["owner"][rid] == r for r in range(world) for rid in mine[r])
    assert min(len(m) for m in mine) >= 80                                   # the router spreads the load
    for o in outs:                                                          # every rank has every stream
        assert all(o["streams"][rid] == _expected_stream(reqs[rid]) for rid in reqs)
        assert o["outstanding_left"] == 0
    assert outs[0]["iterations"] == outs[1]["iterations"] and outs[0]["makespan"] == outs[1]["makespan"]
    assert outs[0]["times"] == outs[1]["times"] and [t[0] for t in outs[0]["times"]] == sorted(reqs)
    ttft = [t[2] - t[1] for t in outs[0]["times"]]
    assert all(np.isfinite(ttft)) and min(ttft) >= 0
    # two ranks finish the trace sooner than one on the same fake executors
    one = b2pa.serve(_trace(), osv.fake_prefill_executor, osv.fake_decode_executor, max_batch_size=8,
                     prefill_chunk_size=256, max_tokens_per_iteration=1536)
    assert outs[0]["makespan"] <= one.makespan_ms


def _saturated_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        reqs = _trace()
        for r in reqs:
            r.arrival_time_ms = 0.0
        res = b2pa.serve(reqs, osv.fake_prefill_executor, osv.fake_decode_executor, max_batch_size=8,
                         prefill_chunk_size=256, max_tokens_per_iteration=1536, device=torch.device("cpu"))
        if rank == 0:
            np.save(os.path.join(out_dir, "sat.npy"), np.array([{"makespan": res.makespan_ms,
                                                                 "streams": res.token_streams}], dtype=object),
                    allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_two_ranks_share_a_saturated_load(tmp_path):
    """Every request arriving at once: each rank serves its share on its own
    clock, so two ranks finish in well under one rank's time (a single shared
    clock advanced by the slower rank's iteration did not)."""
    reqs = _trace()
    for r in reqs:
        r.arrival_time_ms = 0.0
    one = b2pa.serve(reqs, osv.fake_prefill_executor, osv.fake_decode_executor, max_batch_size=8,
                     prefill_chunk_size=256, max_tokens_per_iteration=1536)
    mp.spawn(_saturated_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    two = np.load(tmp_path / "sat.npy", allow_pickle=True)[0]
    assert two["makespan"] < 0.6 * one.makespan_ms
    assert two["streams"] == one.token_streams
