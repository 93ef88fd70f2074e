"""Multi-GPU serving: requests partitioned by sequence across the GPUs of one
node, one continuous-batching scheduler and one set of block pools per rank.

The reference serves from one GPU: ``ContinuousBatchingScheduler.run``
(src/serving/scheduler.py:254-465) admits requests from a FIFO queue by
their simulated arrival time, runs one decode step over every active decode
request, then spends the rest of the iteration's token budget on chunked
prefill of equal-progress groups.  This module runs that policy on every rank
of a ``torch.distributed`` group over the requests routed to the rank:

* ``ContinuousBatchingRank`` -- the reference's policy, stepped one iteration
  (one pass of its loop body, scheduler.py:321-463) at a time, over the
  requests this rank was given;
* ``LeastOutstandingTokensRouter`` -- sends each arriving request to the rank
  with the fewest outstanding tokens (prompt tokens not yet prefilled plus
  tokens not yet generated), ties to the lowest rank.  Every rank evaluates
  it on the same data, so all ranks make the same decisions without a
  message;
* ``serve`` -- the loop.  Per iteration each rank runs one iteration of its
  own scheduler (its requests' attention and KV appends touch only its own
  pools: no collective on that path), then the ranks exchange, in two
  collectives, the token ids they sampled and a small vector of statistics
  (virtual clock, outstanding tokens, completed requests) -- the only
  traffic between GPUs.  Each rank keeps its own virtual clock, advanced by
  its measured runtime as the reference's is (the ranks run in parallel);
  a request is routed once every rank's clock has passed its arrival, and a
  rank with nothing to do moves its clock on to the next arrival.

With one rank ``serve`` reproduces the reference's ``run`` event for event
(the router hands every request to rank 0 up front and the rank's own
arrival rules apply).

Requests and executors are the reference's (``InferenceRequest``,
``run_prefill_chunk`` / ``run_decode_step`` from src/serving/
continuous_generate.py:83-276, or anything with the same contract): an
executor advances the requests it is given and returns a dict with
``batch_runtime_ms``, ``requests_completed`` and ``tokens_scheduled``.
"""
from __future__ import annotations

import bisect
import math
from dataclasses import dataclass, field

import numpy as np
import torch


def outstanding_tokens(request) -> int:
    """Prompt tokens not yet prefilled plus tokens not yet generated."""
    return (max(request.prompt_len - request.prompt_tokens_processed, 0)
            + max(request.max_new_tokens - len(request.generated_token_ids), 0))


class LeastOutstandingTokensRouter:
    """Routes each request to the rank with the fewest outstanding tokens.

    ``sync`` installs the ranks' own counts after an exchange; between
    exchanges ``route`` adds each routed request's tokens to its rank's
    count, so a burst of arrivals spreads over the ranks."""

    def __init__(self, world: int):
        self.world = world
        self.outstanding = np.zeros(world, dtype=np.int64)

    def sync(self, per_rank) -> None:
        self.outstanding[:] = np.asarray(per_rank, dtype=np.int64)

    def route(self, request) -> int:
        r = int(np.argmin(self.outstanding))  # first minimum: ties go to the lowest rank
        self.outstanding[r] += request.prompt_len + request.max_new_tokens
        return r


class ContinuousBatchingRank:
    """The reference's continuous-batching policy over one rank's requests,
    one iteration per ``iterate`` call (src/serving/scheduler.py:254-465:
    FIFO admission by arrival time up to ``max_batch_size`` active requests,
    decode first, then chunked prefill of the largest equal-progress group --
    ties to the earliest arrival -- while the token budget lasts)."""

    def __init__(self, max_batch_size: int, prefill_chunk_size: int, max_tokens_per_iteration: int):
        self.max_batch_size = max_batch_size
        self.prefill_chunk_size = prefill_chunk_size
        self.max_tokens_per_iteration = max_tokens_per_iteration
        self.inbox: list = []       # routed here, not yet enqueued (arrival order)
        self.waiting: list = []
        self.active: list = []
        self.completed: list = []
        self.events: list[dict] = []
        self.event_id = 0
        self._reported: dict[int, int] = {}  # request id -> tokens already reported
        self._owned: list = []

    # ------------------------------------------------------------ requests
    def assign(self, request) -> None:
        keys = [r.arrival_time_ms for r in self.inbox]
        self.inbox.insert(bisect.bisect_right(keys, request.arrival_time_ms), request)
        self._owned.append(request)
        self._reported[request.request_id] = len(request.generated_token_ids)

    def has_work(self) -> bool:
        return bool(self.inbox or self.waiting or self.active)

    def outstanding_tokens(self) -> int:
        return sum(outstanding_tokens(r) for r in self.inbox + self.waiting + self.active)

    def take_new_tokens(self) -> list[tuple[int, int]]:
        """(request id, token id) of every token generated since the last
        call, request by request in generation order."""
        out = []
        for r in self._owned:
            done = self._reported[r.request_id]
            gen = r.generated_token_ids
            if len(gen) > done:
                out.extend((r.request_id, int(t)) for t in gen[done:])
                self._reported[r.request_id] = len(gen)
        return out

    # -------------------------------------------------------------- policy
    def _enqueue(self, now: float) -> None:
        while self.inbox and self.inbox[0].arrival_time_ms <= now:
            self.waiting.append(self.inbox.pop(0))

    def _admit(self) -> None:
        while self.waiting and len(self.active) < self.max_batch_size:
            self.active.append(self.waiting.pop(0))

    def _finish(self, result: dict, release) -> None:
        for done in result["requests_completed"]:
            if release is not None:
                release(done)
            self.active.remove(done)
            self.completed.append(done)

    def _record(self, result: dict, now: float, group: list) -> None:
        self.events.append({"batch_id": self.event_id, "phase": result.get("phase"),
                            "request_ids": [r.request_id for r in group],
                            "dispatch_time_ms": now - result["batch_runtime_ms"], "finish_time_ms": now,
                            "batch_runtime_ms": result["batch_runtime_ms"],
                            "tokens_scheduled": result["tokens_scheduled"],
                            "batch_size": result.get("batch_size")})
        self.event_id += 1

    def iterate(self, now: float, prefill_executor, decode_executor, release=None) -> float:
        """One pass of the reference's scheduling loop starting at virtual
        time ``now``; returns the time after it."""
        if not self.waiting and not self.active and self.inbox:
            now = max(now, self.inbox[0].arrival_time_ms)
        self._enqueue(now)
        self._admit()
        if not self.active:
            return now
        used = 0
        decode_group = [r for r in self.active if r.phase == "decode"]
        if decode_group:
            res = decode_executor(decode_group, now, self.event_id)
            now += res["batch_runtime_ms"]
            used += res["tokens_scheduled"]
            self._finish(res, release)
            self._record(res, now, decode_group)
            self._enqueue(now)
            self._admit()
        budget = max(self.max_tokens_per_iteration - used, 0)
        while budget > 0:
            groups: dict[int, list] = {}
            for r in self.active:
                if r.phase == "prefill":
                    groups.setdefault(r.prompt_tokens_processed, []).append(r)
            if not groups:
                break
            key = max(groups, key=lambda k: (len(groups[k]), -min(r.arrival_time_ms for r in groups[k])))
            group = groups[key]
            group_budget = min(self.prefill_chunk_size, max(budget // max(len(group), 1), 0))
            if group_budget <= 0:
                break
            res = prefill_executor(group, group_budget, now, self.event_id)
            now += res["batch_runtime_ms"]
            budget -= res["tokens_scheduled"]
            self._finish(res, release)
            self._record(res, now, group)
            self._enqueue(now)
            self._admit()
        return now


@dataclass
class ServeResult:
    """What ``serve`` returns on every rank."""

    completed: list                      # this rank's requests, by request id
    events: list                         # this rank's executor calls
    token_streams: dict = field(default_factory=dict)   # request id -> generated ids (all ranks' requests)
    owner: dict = field(default_factory=dict)           # request id -> rank that served it
    iterations: int = 0
    makespan_ms: float = 0.0


def _world(group) -> tuple[int, int]:
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def serve(requests: list, prefill_executor, decode_executor, release=None, *, max_batch_size: int,
          prefill_chunk_size: int, max_tokens_per_iteration: int, group=None,
          device: torch.device | None = None) -> ServeResult:
    """Serves ``requests`` (the same list, in the same order, on every rank)
    with one continuous-batching scheduler per rank of ``group`` (the
    default process group, or a single process without one).  ``device`` is
    where the exchange tensors live: the rank's GPU for NCCL, the CPU for
    gloo (default: this rank's current CUDA device if CUDA is available)."""
    world, rank = _world(group)
    requests = sorted(requests, key=lambda r: r.arrival_time_ms)
    sched = ContinuousBatchingRank(max_batch_size, prefill_chunk_size, max_tokens_per_iteration)
    router = LeastOutstandingTokensRouter(world)
    result = ServeResult(completed=sched.completed, events=sched.events)
    if world == 1:
        for r in requests:
            router.route(r)
            sched.assign(r)
            result.owner[r.request_id] = 0
        now = 0.0
        while len(sched.completed) < len(requests):
            now = sched.iterate(now, prefill_executor, decode_executor, release)
            result.iterations += 1
        for rid, tok in sched.take_new_tokens():
            result.token_streams.setdefault(rid, []).append(tok)
        sched.completed.sort(key=lambda r: r.request_id)
        result.makespan_ms = now
        return result

    import torch.distributed as dist

    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    cap = 4 * max_batch_size  # tokens one rank can emit in one iteration (at most 2 per active slot)
    NS = 5                    # statistics per rank: clock, outstanding tokens, completed, tokens emitted, active
    tok_out = torch.empty(world * cap * 2, dtype=torch.int64, device=device)
    stat_out = torch.empty(world * NS, dtype=torch.float64, device=device)
    nxt, clock, total_done = 0, 0.0, 0
    clocks = np.zeros(world)
    for r in requests:
        result.token_streams[r.request_id] = []
    while total_done < len(requests):
        # Route the requests every rank's clock has passed (all ranks see the
        # same clocks from the last exchange, so all route alike).
        horizon = float(clocks.min())
        while nxt < len(requests) and requests[nxt].arrival_time_ms <= horizon:
            owner = router.route(requests[nxt])
            result.owner[requests[nxt].request_id] = owner
            if owner == rank:
                sched.assign(requests[nxt])
            nxt += 1
        if sched.has_work():
            clock = sched.iterate(clock, prefill_executor, decode_executor, release)
        elif nxt < len(requests):
            # idle: move on to the next arrival, so that routing can proceed
            clock = max(clock, requests[nxt].arrival_time_ms)
        new = sched.take_new_tokens()
        if len(new) > cap:
            raise RuntimeError(f"b2pa.serve: {len(new)} tokens in one iteration exceed the exchange size {cap}")
        mine = torch.full((cap, 2), -1, dtype=torch.int64)
        if new:
            mine[: len(new)] = torch.tensor(new, dtype=torch.int64)
        # the two exchanges of an iteration: sampled tokens, then statistics
        dist.all_gather_into_tensor(tok_out, mine.reshape(-1).to(device), group=group)
        stats = torch.tensor([clock, float(sched.outstanding_tokens()), float(len(sched.completed)), float(len(new)),
                              float(sched.has_work())], dtype=torch.float64)
        dist.all_gather_into_tensor(stat_out, stats.to(device), group=group)
        toks = tok_out.view(world, cap, 2).cpu().numpy()
        st = stat_out.view(world, NS).cpu().numpy()
        for w in range(world):
            for rid, tok in toks[w, : int(st[w, 3])]:
                result.token_streams[int(rid)].append(int(tok))
        clocks = st[:, 0].copy()
        # a rank with nothing to do does not hold routing back
        busy = st[:, 4] > 0
        if nxt < len(requests) and not busy.all():
            clocks[~busy] = np.maximum(clocks[~busy], min(requests[nxt].arrival_time_ms, clocks[busy].max())
                                       if busy.any() else requests[nxt].arrival_time_ms)
        router.sync(st[:, 1])
        total_done = int(st[:, 2].sum())
        result.iterations += 1
    sched.completed.sort(key=lambda r: r.request_id)
    result.makespan_ms = float(clocks.max())
    return result


def gather_request_times(completed: list, group=None) -> list[tuple[int, float, float, float]]:
    """(request id, arrival, first-token time, finish time) of every rank's
    completed requests, on every rank, by request id -- for TTFT and latency
    statistics after a run (one exchange, off the serving loop)."""
    mine = [(r.request_id, r.arrival_time_ms,
             math.nan if r.first_token_time_ms is None else r.first_token_time_ms,
             math.nan if r.finish_time_ms is None else r.finish_time_ms) for r in completed]
    world, _ = _world(group)
    if world == 1:
        return sorted(mine)
    import torch.distributed as dist

    parts = [None] * world
    dist.all_gather_object(parts, mine, group=group)
    return sorted(x for p in parts for x in p)
