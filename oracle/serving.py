"""Restatement of the reference's serving path for BASELINE config[3] --
TEST INFRASTRUCTURE ONLY (used by tests/ to drive the b2pa backend through
the reference's continuous-batching policy on the GPU box, where the
reference itself is not available).

Restates, without importing:
  src/serving/loadgen.py:14-85          generate_requests (same RNG draws)
  src/serving/request.py:6-60           InferenceRequest
  src/serving/scheduler.py:254-465      ContinuousBatchingScheduler.run
  src/serving/continuous_generate.py    run_prefill_chunk (:83-194),
                                        run_decode_step (:198-276)
  src/serving/metrics.py:4-16,43-49     percentile, throughput_tokens_per_s
The scheduler and the load generator are pinned to the reference by
tests/test_serving_harness.py (golden vectors from the reference's own run with
the deterministic fake executors defined here).
"""
from __future__ import annotations

import random
import time
from dataclasses import dataclass, field

import torch
from torch.nn.utils.rnn import pad_sequence


@dataclass(frozen=True)
class WorkloadProfile:
    name: str
    prompt_len_min: int
    prompt_len_max: int
    max_new_tokens_min: int
    max_new_tokens_max: int
    weight: float


# BASELINE config[3] request mix.
CONFIG3_PROFILES = [
    WorkloadProfile("short_qa", 32, 128, 16, 64, 0.4),
    WorkloadProfile("chat_turn", 128, 384, 64, 192, 0.3),
    WorkloadProfile("rag_answer", 512, 832, 32, 128, 0.2),
    WorkloadProfile("long_summary", 640, 896, 64, 128, 0.1),
]


@dataclass
class Request:
    request_id: int
    arrival_time_ms: float
    prompt_len: int
    max_new_tokens: int
    prompt_ids: torch.Tensor
    workload_name: str = "fixed"
    start_time_ms: float | None = None
    finish_time_ms: float | None = None
    batch_id: int | None = None
    phase: str = "prefill"
    prompt_tokens_processed: int = 0
    generated_token_ids: list = field(default_factory=list)
    kv_caches: list | None = None
    first_token_time_ms: float | None = None

    @property
    def num_generated_tokens(self) -> int:
        return len(self.generated_token_ids)

    @property
    def first_token_latency_ms(self) -> float:
        return 0.0 if self.first_token_time_ms is None else self.first_token_time_ms - self.arrival_time_ms

    @property
    def latency_ms(self) -> float:
        return 0.0 if self.finish_time_ms is None else self.finish_time_ms - self.arrival_time_ms


def generate_requests(num_requests: int, arrival_rate_rps: float, vocab_size: int, profiles, seed: int = 42):
    """Poisson arrivals (exponential gaps), profile by weight, lengths uniform
    in the profile ranges, prompt ids uniform -- in the reference's draw order."""
    rng = random.Random(seed)
    gen = torch.Generator().manual_seed(seed)
    weights = [p.weight for p in profiles]
    now = 0.0
    mean_gap = 1000.0 / arrival_rate_rps
    out = []
    for rid in range(num_requests):
        if rid > 0:
            now += rng.expovariate(1.0 / mean_gap)
        prof = rng.choices(profiles, weights=weights, k=1)[0]
        plen = rng.randint(prof.prompt_len_min, prof.prompt_len_max)
        nnew = rng.randint(prof.max_new_tokens_min, prof.max_new_tokens_max)
        ids = torch.randint(low=0, high=vocab_size, size=(plen,), generator=gen)
        out.append(Request(rid, now, plen, nnew, ids, prof.name))
    return out


def percentile(values, p: float) -> float:
    if not values:
        return 0.0
    values = sorted(values)
    if len(values) == 1:
        return values[0]
    rank = (len(values) - 1) * (p / 100.0)
    lo = int(rank)
    hi = min(lo + 1, len(values) - 1)
    w = rank - lo
    return values[lo] * (1.0 - w) + values[hi] * w


def throughput_tokens_per_s(completed) -> float:
    if not completed:
        return 0.0
    makespan = max(r.finish_time_ms for r in completed) - min(r.arrival_time_ms for r in completed)
    total = sum(r.max_new_tokens for r in completed)
    return total / (makespan / 1000.0) if makespan > 0 else 0.0


class ContinuousScheduler:
    """Decode-first continuous batching with chunked prefill under a
    per-iteration token budget; requests grouped by equal prompt progress."""

    def __init__(self, max_batch_size: int, prefill_chunk_size: int, max_tokens_per_iteration: int):
        self.max_batch_size = max_batch_size
        self.prefill_chunk_size = prefill_chunk_size
        self.max_tokens_per_iteration = max_tokens_per_iteration

    @staticmethod
    def _enqueue(requests, nxt, now, waiting):
        while nxt < len(requests) and requests[nxt].arrival_time_ms <= now:
            waiting.append(requests[nxt])
            nxt += 1
        return nxt

    def _admit(self, waiting, active):
        while waiting and len(active) < self.max_batch_size:
            active.append(waiting.pop(0))

    @staticmethod
    def _groups(active):
        g = {}
        for r in active:
            if r.phase == "prefill":
                g.setdefault(r.prompt_tokens_processed, []).append(r)
        return g

    @staticmethod
    def _pick(groups):
        return max(groups, key=lambda k: (len(groups[k]), -min(r.arrival_time_ms for r in groups[k])))

    def run(self, requests, prefill_executor, decode_executor, release=None):
        requests = sorted(requests, key=lambda r: r.arrival_time_ms)
        waiting, active, completed, events = [], [], [], []
        now, nxt, eid = 0.0, 0, 0
        while len(completed) < len(requests):
            if not waiting and not active and nxt < len(requests):
                now = max(now, requests[nxt].arrival_time_ms)
            nxt = self._enqueue(requests, nxt, now, waiting)
            self._admit(waiting, active)
            if not active:
                continue
            used = 0
            dec = [r for r in active if r.phase == "decode"]
            if dec:
                res = decode_executor(dec, now, eid)
                now += res["batch_runtime_ms"]
                used += res["tokens_scheduled"]
                for done in res["requests_completed"]:
                    if release is not None:
                        release(done)
                    active.remove(done)
                    completed.append(done)
                events.append(("decode", [r.request_id for r in dec], now - res["batch_runtime_ms"],
                               res["batch_runtime_ms"], res["tokens_scheduled"]))
                eid += 1
                nxt = self._enqueue(requests, nxt, now, waiting)
                self._admit(waiting, active)
            budget = max(self.max_tokens_per_iteration - used, 0)
            if budget <= 0:
                continue
            while budget > 0:
                groups = self._groups(active)
                if not groups:
                    break
                group = groups[self._pick(groups)]
                gb = min(self.prefill_chunk_size, max(budget // max(len(group), 1), 0))
                if gb <= 0:
                    break
                res = prefill_executor(group, gb, now, eid)
                now += res["batch_runtime_ms"]
                budget -= res["tokens_scheduled"]
                for done in res["requests_completed"]:
                    if release is not None:
                        release(done)
                    active.remove(done)
                    completed.append(done)
                events.append(("prefill", [r.request_id for r in group], now - res["batch_runtime_ms"],
                               res["batch_runtime_ms"], res["tokens_scheduled"]))
                eid += 1
                nxt = self._enqueue(requests, nxt, now, waiting)
                self._admit(waiting, active)
        completed.sort(key=lambda r: r.request_id)
        return completed, events


# ------------------------------------------------------------- executors
def _finish_prefill(requests, chunk_start, chunk_lengths, start_ms, finish_ms, event_id, next_tokens):
    done = []
    for i, r in enumerate(requests):
        if r.start_time_ms is None:
            r.start_time_ms, r.batch_id = start_ms, event_id
        r.prompt_tokens_processed = chunk_start + chunk_lengths[i]
        if r.prompt_tokens_processed >= r.prompt_len:
            r.generated_token_ids.append(int(next_tokens[i]))
            if r.first_token_time_ms is None:
                r.first_token_time_ms = finish_ms
            if r.num_generated_tokens >= r.max_new_tokens:
                r.phase, r.finish_time_ms = "finished", finish_ms
                done.append(r)
            else:
                r.phase = "decode"
        else:
            r.phase = "prefill"
    return done


def _finish_decode(requests, start_ms, finish_ms, event_id, next_tokens):
    done = []
    for i, r in enumerate(requests):
        if r.start_time_ms is None:
            r.start_time_ms, r.batch_id = start_ms, event_id
        r.generated_token_ids.append(int(next_tokens[i]))
        if r.num_generated_tokens >= r.max_new_tokens:
            r.phase, r.finish_time_ms = "finished", finish_ms
            done.append(r)
        else:
            r.phase = "decode"
    return done


def fake_prefill_executor(requests, chunk_size, start_ms, event_id):
    """Deterministic stand-in for run_prefill_chunk (no model): runtime
    0.5 ms + 2 us per scheduled token; the emitted token is request_id % 97."""
    cs = requests[0].prompt_tokens_processed
    lens = [max(min(chunk_size, r.prompt_len - cs), 0) for r in requests]
    if max(lens) <= 0:
        return {"batch_runtime_ms": 0.0, "requests_completed": [], "tokens_scheduled": 0}
    rt = 0.5 + 0.002 * sum(lens)
    done = _finish_prefill(requests, cs, lens, start_ms, start_ms + rt, event_id,
                           [r.request_id % 97 for r in requests])
    return {"batch_runtime_ms": rt, "requests_completed": done, "tokens_scheduled": sum(lens),
            "batch_size": len(requests), "phase": "prefill", "prompt_len": max(r.prompt_len for r in requests),
            "max_new_tokens": max(r.max_new_tokens for r in requests)}


def fake_decode_executor(requests, start_ms, event_id):
    """Deterministic stand-in for run_decode_step: 0.3 ms + 0.05 ms per request."""
    rt = 0.3 + 0.05 * len(requests)
    done = _finish_decode(requests, start_ms, start_ms + rt, event_id, [r.request_id % 89 for r in requests])
    return {"batch_runtime_ms": rt, "requests_completed": done, "tokens_scheduled": len(requests),
            "batch_size": len(requests), "phase": "decode", "prompt_len": max(r.prompt_len for r in requests),
            "max_new_tokens": max(r.max_new_tokens for r in requests)}


class ModelExecutors:
    """run_prefill_chunk / run_decode_step for a model of oracle/model.py:
    request caches created on first use, stacked per layer into a batch object
    around the same states every call, runtime measured with a device sync on
    both sides (src/utils/timing.py:11-21)."""

    def __init__(self, model, device):
        self.model = model
        self.device = device

    def _sync(self):
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def _caches(self, requests):
        missing = [i for i, r in enumerate(requests) if r.kv_caches is None]
        if missing:
            created = self.model.create_request_kv_caches(len(missing))
            for j, i in enumerate(missing):
                requests[i].kv_caches = created[j]
        nl = len(requests[0].kv_caches)
        bc = self.model.backend.batch_cls
        return [bc(states=[r.kv_caches[l] for r in requests], pool=requests[0].kv_caches[l].pool) for l in range(nl)]

    @torch.no_grad()
    def prefill(self, requests, chunk_size, start_ms, event_id):
        cs = requests[0].prompt_tokens_processed
        lens = [max(min(chunk_size, r.prompt_len - cs), 0) for r in requests]
        if max(lens) <= 0:
            return {"batch_runtime_ms": 0.0, "requests_completed": [], "tokens_scheduled": 0}
        batch = pad_sequence([r.prompt_ids[cs:cs + n].to(self.device) for r, n in zip(requests, lens)],
                             batch_first=True, padding_value=0)
        cur = torch.tensor(lens, device=self.device, dtype=torch.long)
        caches = self._caches(requests)
        self._sync()
        t0 = time.perf_counter()
        logits, _ = self.model(batch, kv_caches=caches, position_offset=cs, current_lengths=cur)
        self._sync()
        rt = (time.perf_counter() - t0) * 1000.0
        last = logits[torch.arange(len(requests), device=self.device), cur - 1, :]
        nxt = torch.argmax(last, dim=-1).tolist()
        done = _finish_prefill(requests, cs, lens, start_ms, start_ms + rt, event_id, nxt)
        return {"batch_runtime_ms": rt, "requests_completed": done, "tokens_scheduled": sum(lens)}

    @torch.no_grad()
    def decode(self, requests, start_ms, event_id):
        inp = torch.tensor([[r.generated_token_ids[-1]] for r in requests], device=self.device, dtype=torch.long)
        pos = torch.tensor([r.prompt_len + r.num_generated_tokens - 1 for r in requests], device=self.device,
                           dtype=torch.long)
        caches = self._caches(requests)
        self._sync()
        t0 = time.perf_counter()
        logits, _ = self.model(inp, kv_caches=caches, position_offset=pos)
        self._sync()
        rt = (time.perf_counter() - t0) * 1000.0
        nxt = torch.argmax(logits[:, -1, :], dim=-1).tolist()
        done = _finish_decode(requests, start_ms, start_ms + rt, event_id, nxt)
        return {"batch_runtime_ms": rt, "requests_completed": done, "tokens_scheduled": len(requests)}

    def release(self, request):
        for c in request.kv_caches or []:
            c.release()
