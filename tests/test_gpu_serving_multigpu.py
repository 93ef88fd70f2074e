"""BASELINE config[3] on several GPUs of one node (b2pa.serve): the
200-request trace (52 req/s, the config[3] mix, seed 42) on the config[0]
model with the b2pa backend, one rank per GPU over NCCL, each rank with its
own scheduler and block pools; ranks exchange only the sampled token ids and
a few statistics per iteration.  Runs N = 1 and every N in (2, 4, 8) the
node has GPUs for; needs at least two GPUs.

Checks: every request completes on exactly one rank with its token budget,
and every request's token stream is identical to the one-GPU run.  Prints
tokens/s and p50/p99 time to first token per N (virtual clock advanced by
measured GPU time, as the reference's scheduler does).  A second, saturated
run -- the same requests all arriving at once, decode steps on
b2pa.FusedDecodeExecutor -- shows how throughput scales with N when arrivals
do not bound it; its tokens must equal the first run's too."""
from __future__ import annotations

import json
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    import torch.distributed as dist

    import b2pa
    from oracle import model as om
    from oracle import serving as osv

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    if world > 1:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    try:
        prev = b2pa.set_fused_append(True)
        model, _ = om.config0_model(om.b2pa_backend(), dev)
        ex = osv.ModelExecutors(model, dev)
        # warm-up on this rank alone, as the reference's harness does
        # (experiments/batching/benchmark_scheduler.py:43-61)
        warm = osv.generate_requests(8, 1000.0, 5000, [osv.WorkloadProfile("w", 256, 256, 2, 2, 1.0)], seed=1)
        osv.ContinuousScheduler(8, 256, 1536).run(warm, ex.prefill, ex.decode, ex.release)
        model.pools = None
        reqs = osv.generate_requests(200, 52.0, 5000, osv.CONFIG3_PROFILES, seed=42)
        res = b2pa.serve(reqs, ex.prefill, ex.decode, ex.release, max_batch_size=8, prefill_chunk_size=256,
                         max_tokens_per_iteration=1536, device=dev)
        times = b2pa.gather_request_times(res.completed)
        assert all(r.num_generated_tokens == r.max_new_tokens for r in res.completed)
        assert b2pa.read_status(dev) == 0
        b2pa.set_fused_append(prev)
        # saturated: the same request mix all arriving at once, decode steps on b2pa.FusedDecodeExecutor
        prev = b2pa.set_fused_append(True)
        model_s, _ = om.config0_model(om.b2pa_backend(), dev)
        ex_s = osv.ModelExecutors(model_s, dev)
        fused = b2pa.FusedDecodeExecutor(model_s, dev, max_batch=8)
        osv.ContinuousScheduler(8, 256, 1536).run(
            osv.generate_requests(8, 1000.0, 5000, [osv.WorkloadProfile("w", 256, 256, 3, 3, 1.0)], seed=1),
            ex_s.prefill, fused, ex_s.release)
        model_s.pools = None
        sat = osv.generate_requests(200, 52.0, 5000, osv.CONFIG3_PROFILES, seed=42)
        for r in sat:
            r.arrival_time_ms = 0.0
        res_s = b2pa.serve(sat, ex_s.prefill, fused, ex_s.release, max_batch_size=8, prefill_chunk_size=256,
                           max_tokens_per_iteration=1536, device=dev)
        times_s = b2pa.gather_request_times(res_s.completed)
        assert b2pa.read_status(dev) == 0
        b2pa.set_fused_append(prev)
        if rank == 0:
            budget = {r.request_id: r.max_new_tokens for r in reqs}

            def summary(rs, tm):
                ttft = [ft - a for _, a, ft, _ in tm]
                makespan = max(f for *_, f in tm) - min(a for _, a, _, _ in tm)
                return {"completed": len(tm),
                        "per_rank_requests": [sum(1 for o in rs.owner.values() if o == w) for w in range(world)],
                        "throughput_tokens_per_s": sum(budget.values()) / (makespan / 1000.0),
                        "ttft_p50_ms": osv.percentile(ttft, 50), "ttft_p99_ms": osv.percentile(ttft, 99),
                        "makespan_ms": makespan, "iterations": rs.iterations,
                        "streams": {str(k): v for k, v in rs.token_streams.items()}}

            out = {"n_gpus": world, **summary(res, times), "saturated_fused_decode": summary(res_s, times_s)}
            with open(os.path.join(out_dir, f"serve_n{world}.json"), "w") as f:
                json.dump(out, f)
    finally:
        if world > 1:
            dist.destroy_process_group()


def _run(world: int, out_dir: str) -> dict:
    mp.spawn(_worker, args=(world, _free_port(), out_dir), nprocs=world, join=True)
    with open(os.path.join(out_dir, f"serve_n{world}.json")) as f:
        return json.load(f)


def test_config3_trace_on_several_gpus(tmp_path):
    n_dev = torch.cuda.device_count()
    if n_dev < 2:
        pytest.skip("needs at least two GPUs")
    def brief(res):
        out = {k: v for k, v in res.items() if k not in ("streams", "saturated_fused_decode")}
        out["saturated_fused_decode"] = {k: v for k, v in res["saturated_fused_decode"].items() if k != "streams"}
        return out

    one = _run(1, str(tmp_path))
    assert one["completed"] == 200 and one["saturated_fused_decode"]["completed"] == 200
    # the saturated run's decode steps are on the fused executor: same tokens as the model's own steps
    assert one["saturated_fused_decode"]["streams"] == one["streams"]
    report = [brief(one)]
    for world in (2, 4, 8):
        if world > n_dev:
            break
        res = _run(world, str(tmp_path))
        for run in (res, res["saturated_fused_decode"]):
            assert run["completed"] == 200
            assert sum(run["per_rank_requests"]) == 200 and min(run["per_rank_requests"]) > 0
            differ = [k for k in one["streams"] if one["streams"][k] != run["streams"][k]]
            assert not differ, f"{len(differ)} requests' token streams differ from the one-GPU run: {differ[:5]}"
        report.append(brief(res))
    print(json.dumps(report))
