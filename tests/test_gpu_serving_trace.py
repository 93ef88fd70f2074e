"""BASELINE config[3] on the GPU: the 200-request continuous-batching trace
(52 req/s, the config[3] mix, seed 42) through the reference's scheduling
policy (restated in oracle/serving.py, pinned on CPU) on the config[0] model
with the b2pa backend.  Every request completes with its token budget; one
attention call in eight is shadowed by the torch restatement of the
reference's attention on the same inputs (rtol 1e-4 / atol 1e-5).  Reports
tokens/s and p50/p99 time to first token, the virtual clock advanced by
measured GPU time as in the reference."""
from __future__ import annotations

import json
import time

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import serving as osv
from oracle import torch_paged as tp

pytestmark = pytest.mark.gpu


def _warm(ex):
    # warm-up as the reference's harness does (experiments/batching/benchmark_scheduler.py:43-61)
    warm = osv.generate_requests(8, 1000.0, 5000, [osv.WorkloadProfile("w", 256, 256, 2, 2, 1.0)], seed=1)
    osv.ContinuousScheduler(8, 256, 1536).run(warm, ex.prefill, ex.decode, ex.release)


def _complete(done):
    assert len(done) == 200
    assert all(r.num_generated_tokens == r.max_new_tokens for r in done)


def test_config3_serving_trace(cuda_device):
    import b2pa

    base = om.b2pa_backend()
    shadow = {"n": 0, "checked": 0, "max_err": 0.0}

    def attention(q, kv, cur):
        out = base.attention(q, kv, cur)
        shadow["n"] += 1
        if shadow["n"] % 8 == 1:
            ref = tp.paged_attention_torch(q, kv, cur)
            np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), rtol=1e-4, atol=1e-5)
            shadow["checked"] += 1
            shadow["max_err"] = max(shadow["max_err"], float((out - ref).abs().max()))
        return out

    backend = om.Backend("b200_paged", base.pool_cls, base.state_cls, base.batch_cls, attention)
    model, _ = om.config0_model(backend, cuda_device)
    ex = osv.ModelExecutors(model, cuda_device)
    _warm(ex)
    # pass 1: parity -- shadow-check one attention call in eight, with the
    # decode append as a separate kernel and fused into the decode launch
    for fused in (False, True):
        prev = b2pa.set_fused_append(fused)
        try:
            model.pools = None
            reqs = osv.generate_requests(200, 52.0, 5000, osv.CONFIG3_PROFILES, seed=42)
            done, _ = osv.ContinuousScheduler(8, 256, 1536).run(reqs, ex.prefill, ex.decode, ex.release)
        finally:
            b2pa.set_fused_append(prev)
        _complete(done)
    assert shadow["checked"] > 200
    # pass 2: timing -- the b2pa attention alone inside the timed model calls
    report = {
        "config": "BASELINE config[3]: 200 requests @52 req/s, config[3] mix, ContinuousBatchingScheduler(8, 256, 1536), "
                  "config[0] model FP32, b2pa backend, one B200",
        "shadow_checked_attention_calls": shadow["checked"], "shadow_max_abs_err": shadow["max_err"],
    }
    for fused in (False, True):
        model_t, _ = om.config0_model(base, cuda_device)
        ex = osv.ModelExecutors(model_t, cuda_device)
        prev = b2pa.set_fused_append(fused)
        try:
            _warm(ex)
            model_t.pools = None
            reqs = osv.generate_requests(200, 52.0, 5000, osv.CONFIG3_PROFILES, seed=42)
            t0 = time.perf_counter()
            done, events = osv.ContinuousScheduler(8, 256, 1536).run(reqs, ex.prefill, ex.decode, ex.release)
            wall = time.perf_counter() - t0
        finally:
            b2pa.set_fused_append(prev)
        _complete(done)
        assert all(r.first_token_time_ms is not None for r in done)
        assert b2pa.read_status(cuda_device) == 0
        ttft = [r.first_token_latency_ms for r in done]
        report["fused_append" if fused else "append_then_decode"] = {
            "throughput_tokens_per_s": osv.throughput_tokens_per_s(done),
            "ttft_p50_ms": osv.percentile(ttft, 50), "ttft_p99_ms": osv.percentile(ttft, 99),
            "latency_p99_ms": osv.percentile([r.latency_ms for r in done], 99),
            "events": len(events), "decode_events": sum(1 for e in events if e[0] == "decode"),
            "virtual_gpu_ms": sum(e[3] for e in events), "wall_s": wall,
        }
    print(json.dumps(report))


def test_config3_trace_fused_decode_executor(cuda_device):
    """The same trace with the decode steps on b2pa.FusedDecodeExecutor (the
    model's non-attention ops on b2pa kernels, one shared block table per
    step) and the prompt chunks on the model: every request completes, and
    every request's tokens equal the run with the model's own decode step."""
    import b2pa

    prev = b2pa.set_fused_append(True)
    streams, report = {}, {"config": "BASELINE config[3] trace, one B200: decode steps on the model vs on "
                                     "b2pa.FusedDecodeExecutor (prefill chunks on the model both ways)"}
    try:
        for mode in ("model_decode", "fused_decode", "model_decode", "fused_decode"):
            model, _ = om.config0_model(om.b2pa_backend(), cuda_device)
            ex = osv.ModelExecutors(model, cuda_device)
            decode = b2pa.FusedDecodeExecutor(model, cuda_device, max_batch=8) if mode == "fused_decode" else ex.decode
            warm = osv.generate_requests(8, 1000.0, 5000, [osv.WorkloadProfile("w", 256, 256, 3, 3, 1.0)], seed=1)
            osv.ContinuousScheduler(8, 256, 1536).run(warm, ex.prefill, decode, ex.release)
            model.pools = None
            reqs = osv.generate_requests(200, 52.0, 5000, osv.CONFIG3_PROFILES, seed=42)
            done, events = osv.ContinuousScheduler(8, 256, 1536).run(reqs, ex.prefill, decode, ex.release)
            _complete(done)
            streams[mode] = {r.request_id: list(r.generated_token_ids) for r in done}
            ttft = [r.first_token_latency_ms for r in done]
            dec = [e[3] for e in events if e[0] == "decode"]
            report[mode] = {"throughput_tokens_per_s": osv.throughput_tokens_per_s(done),
                            "ttft_p50_ms": osv.percentile(ttft, 50), "ttft_p99_ms": osv.percentile(ttft, 99),
                            "decode_step_ms_mean": float(np.mean(dec)), "decode_events": len(dec)}
    finally:
        b2pa.set_fused_append(prev)
    differ = [k for k in streams["model_decode"] if streams["model_decode"][k] != streams["fused_decode"][k]]
    assert not differ, f"{len(differ)} requests' tokens differ: {differ[:5]}"
    assert b2pa.read_status(cuda_device) == 0
    print(json.dumps(report))
