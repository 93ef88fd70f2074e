"""Pins the serving restatement used by the config[3] GPU test
(oracle/serving.py) to the reference's own load generator and continuous
scheduler (golden from the reference run with deterministic fake executors).
CPU only."""
from __future__ import annotations

import numpy as np

from oracle import serving as osv
from tests._helpers import load_golden


def test_load_generator_matches_reference():
    g = load_golden("serving_config3")
    reqs = osv.generate_requests(200, 52.0, 5000, osv.CONFIG3_PROFILES, seed=42)
    np.testing.assert_array_equal(np.array([r.arrival_time_ms for r in reqs]), g["arrival_ms"])
    assert [r.prompt_len for r in reqs] == g["prompt_len"].tolist()
    assert [r.max_new_tokens for r in reqs] == g["max_new_tokens"].tolist()
    assert [int(r.prompt_ids.sum()) for r in reqs] == g["prompt_id_sums"].tolist()
    assert np.array_equal(reqs[0].prompt_ids.numpy(), g["first_prompt"])
    assert [r.workload_name for r in reqs] == g["workload"].tolist()


def test_continuous_scheduler_matches_reference():
    g = load_golden("serving_config3")
    reqs = osv.generate_requests(200, 52.0, 5000, osv.CONFIG3_PROFILES, seed=42)
    sched = osv.ContinuousScheduler(8, 256, 1536)
    done, events = sched.run(reqs, osv.fake_prefill_executor, osv.fake_decode_executor)
    assert [e[0] for e in events] == g["ev_phase"].tolist()
    assert [len(e[1]) for e in events] == g["ev_batch_size"].tolist()
    assert [e[4] for e in events] == g["ev_tokens"].tolist()
    np.testing.assert_allclose([e[2] for e in events], g["ev_dispatch_ms"], rtol=1e-12, atol=1e-9)
    np.testing.assert_allclose([r.first_token_time_ms for r in done], g["first_token_ms"], rtol=1e-12, atol=1e-9)
    np.testing.assert_allclose([r.finish_time_ms for r in done], g["finish_ms"], rtol=1e-12, atol=1e-9)
    ttft = [r.first_token_latency_ms for r in done if r.first_token_time_ms is not None]
    np.testing.assert_allclose([osv.percentile(ttft, 50), osv.percentile(ttft, 99)], g["ttft_p50_p99"], rtol=1e-12)
