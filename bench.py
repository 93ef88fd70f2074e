"""Benchmark of the paged-attention hot path on B200.

Workload (per GPU, weak scaling by default): 512 sequences, context lengths
L ~ U[1024, 8192] (seeded), 32 heads x 128 dims, bf16 K/V in a
[num_blocks, 32, 16, 128] block pool sized to 1.2x the pages, random
non-overlapping block tables, N(0,1) data.  One step = one KV append of a new
token for every sequence + one paged decode over every sequence -- what
CausalSelfAttention.forward does per layer per decode step
(src/model/attention.py:56-62 of the reference).

Arms:
  default            b2pa kernels.  ``value``: device-resident inputs, kernels
                     launched through the C ABI, CUDA-event timed; by default
                     each step is one b2pa_paged_decode_append call (append
                     fused into the decode launch; --decode-append separate
                     times b2pa_kv_append + b2pa_paged_decode).  ``e2e``: the
                     public API (BatchedPagedKVCache.append_batch +
                     paged_attention, with b2pa.set_fused_append unless
                     --decode-append separate) with q/k/v copied from pinned
                     host memory and the output copied back every step.
  --impl reference   the CPU restatement of the reference's torch path
                     (oracle/paged_oracle.c, all host threads) on a bounded
                     sample of the same workload, rank 0 only.

Multi-GPU: launch under torchrun; each rank owns its own pool and sequences
(no collective on the hot path); NCCL only reduces the timings.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "efficient-inference-system_b200"))
sys.path.insert(0, str(REPO))

H, D, BS = 32, 128, 16
LMIN, LMAX = 1024, 8192
POOL_SLACK = 1.2
SEED = 4
# ncu, decode kernel with the fused append, 16-sequence case of this workload:
# (dram read 1.438635e9 + write 6.589696e6) / 1.437325e9 algorithmic bytes
DECODE_TRAFFIC_PER_ALGORITHMIC_BYTE = (1.438635e9 + 6.589696e6) / 1.437325e9


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b2pa", "reference"], default="b2pa")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak")
    ap.add_argument("--seqs", type=int, default=512, help="sequences per GPU (weak) or in total (strong)")
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the end-to-end leg (default: --steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the config[1] / config[2] kernel timings in the main line (N=1)")
    ap.add_argument("--len-range", type=int, nargs=2, default=None, metavar=("LO", "HI"),
                    help="context lengths U[LO,HI] instead of config[4]'s U[1024,8192] (small profiling cases; "
                         "the line then names the range)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU work of the baseline sample")
    ap.add_argument("--decode-append", choices=["separate", "fused"], default="fused",
                    help="separate: b2pa_kv_append then b2pa_paged_decode per step; fused: one "
                         "b2pa_paged_decode_append (e2e: b2pa.set_fused_append)")
    ap.add_argument("--workload", choices=["decode", "prefill", "decode_f32"], default="decode",
                    help="decode: config[4] (default, the headline); prefill: config[2] chunked prefill "
                         "(bf16 and fp32); decode_f32: config[1]")
    return ap.parse_args(argv)


# --------------------------------------------------------------- workload
def all_lengths(total: int, lo: int = LMIN, hi: int = LMAX) -> np.ndarray:
    rng = np.random.default_rng(SEED)
    return rng.integers(lo, hi + 1, size=total)


def balanced_partition(lens: np.ndarray, world: int) -> list[np.ndarray]:
    """Splits sequences over ``world`` ranks with equal counts (to within one)
    and nearly equal token totals: longest first, each to the rank with the
    smallest total among those with room (greedy longest-processing-time) --
    the router a sequence-partitioned deployment uses, since a rank's decode
    time is proportional to the tokens it reads.  Returns each rank's
    indices into ``lens``, ascending."""
    n = len(lens)
    cap = [n // world + (1 if r < n % world else 0) for r in range(world)]
    totals = np.zeros(world, dtype=np.int64)
    count = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in np.argsort(-np.asarray(lens), kind="stable").tolist():
        r = min((r for r in range(world) if count[r] < cap[r]), key=lambda r: (totals[r], r))
        parts[r].append(i)
        count[r] += 1
        totals[r] += int(lens[i])
    return [np.sort(np.asarray(p, dtype=np.int64)) for p in parts]


def my_sequences(args, rank: int, world: int, scaling: str | None = None) -> np.ndarray:
    """Context lengths of this rank's sequences.  Weak scaling: a seeded draw
    of ``seqs * world`` sequences (``seqs`` per GPU); strong: the fixed draw
    of ``seqs``; either way spread over the ranks by ``balanced_partition``."""
    scaling = scaling or args.scaling
    lo, hi = getattr(args, "len_range", None) or (LMIN, LMAX)
    lens = all_lengths(args.seqs * world if scaling == "weak" else args.seqs, lo, hi)
    return lens[balanced_partition(lens, world)[rank]]


def algorithmic_decode_bytes(lens_post: np.ndarray, es: int = 2) -> int:
    """Bytes a decode launch must move: K and V of every visible token, q,
    out, the block-table entries and the two length arrays."""
    B = len(lens_post)
    pages = int(np.sum((lens_post + BS - 1) // BS))
    return int(2 * H * D * es * int(lens_post.sum()) + 2 * B * H * D * es + 4 * pages + 8 * B)


def max_over_ranks(values: list[float], device, world: int) -> list[float]:
    """Element-wise max of per-rank timings (all ranks call it, in the same
    order); identity on one rank."""
    if world == 1:
        return list(values)
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


class Workload:
    """This rank's pool, block tables and per-step metadata, on the device."""

    def __init__(self, torch, dev, lens0: np.ndarray, steps_total: int, rank: int):
        self.B = len(lens0)
        self.lens0 = lens0.astype(np.int64)
        final = self.lens0 + steps_total
        pages0 = (self.lens0 + BS - 1) // BS
        pages_final = (final + BS - 1) // BS
        self.num_blocks = int(math.ceil(POOL_SLACK * int(pages0.sum())))
        assert int(pages_final.sum()) <= self.num_blocks
        rng = np.random.default_rng(SEED * 1000 + rank)
        perm = rng.permutation(self.num_blocks).astype(np.int32)
        self.max_pages = int(pages_final.max())
        table = np.full((self.B, self.max_pages), -1, dtype=np.int32)
        o = 0
        for b in range(self.B):
            n = int(pages_final[b])
            table[b, :n] = perm[o:o + n]
            o += n
        self.table = table
        self.used_blocks = o
        gen = torch.Generator(device=dev).manual_seed(SEED + rank)
        shape = (self.num_blocks, H, BS, D)
        self.k_pool = torch.randn(shape, generator=gen, device=dev, dtype=torch.bfloat16)
        self.v_pool = torch.randn(shape, generator=gen, device=dev, dtype=torch.bfloat16)
        self.page_table = torch.from_numpy(table).to(dev)
        steps = np.arange(steps_total, dtype=np.int64)
        start = self.lens0[None, :] + steps[:, None]                       # [S, B]
        self.start_pos = torch.from_numpy(start.astype(np.int32)).to(dev)
        self.seq_lens = torch.from_numpy((start + 1).astype(np.int32)).to(dev)
        self.ones = torch.ones(self.B, dtype=torch.int32, device=dev)
        x = torch.randn(self.B, 1, 3, H, D, generator=gen, device=dev, dtype=torch.bfloat16)
        self.k_new = x[:, :, 0].transpose(1, 2)                             # strided [B,H,1,D] views
        self.v_new = x[:, :, 1].transpose(1, 2)
        self.q = x[:, :, 2].transpose(1, 2)
        self.out = torch.empty_like(self.q)

    def pool_bytes(self) -> int:
        return 2 * self.k_pool.numel() * 2


def run_device_steps(torch, lib, _lib, wl: Workload, dev, first_step: int, n: int, decode_events=None,
                     fused: bool = False):
    """n steps of (append, decode) through the C ABI, inputs resident; with
    ``fused`` each step is one b2pa_paged_decode_append call (decode_events
    then bracket that call)."""
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    status = _lib.status_buffer(dev).data_ptr()
    ws_bytes = lib.b2pa_paged_decode_workspace_size(wl.B, H, D, wl.max_pages, BS, _lib.DTYPE_BF16)
    ws = _lib.workspace(dev, ws_bytes)
    s_new = _lib.strides4(wl.k_new)
    s_v = _lib.strides4(wl.v_new)
    s_pool = _lib.strides4(wl.k_pool)
    s_q = _lib.strides4(wl.q)
    s_out = _lib.strides4(wl.out)
    scale = 1.0 / math.sqrt(D)
    s_k = _lib.strides4(wl.k_new)
    for i in range(n):
        s = first_step + i
        if fused:
            if decode_events is not None:
                decode_events[i][0].record(stream)
            rc = lib.b2pa_paged_decode_append(
                wl.q.data_ptr(), s_q, wl.k_new.data_ptr(), s_k, wl.v_new.data_ptr(), s_v, wl.k_pool.data_ptr(),
                wl.v_pool.data_ptr(), s_pool, wl.num_blocks, wl.page_table.data_ptr(), wl.max_pages, wl.max_pages,
                wl.seq_lens[s].data_ptr(), wl.ones.data_ptr(), wl.start_pos[s].data_ptr(), wl.ones.data_ptr(), None,
                wl.out.data_ptr(), s_out, wl.B, H, D, BS, scale, _lib.DTYPE_BF16, ws.data_ptr(), ws.numel(),
                status, sh)
            _lib.check(rc, "b2pa_paged_decode_append")
            if decode_events is not None:
                decode_events[i][1].record(stream)
            continue
        rc = lib.b2pa_kv_append(wl.k_new.data_ptr(), s_new, wl.v_new.data_ptr(), s_v, wl.k_pool.data_ptr(),
                                wl.v_pool.data_ptr(), s_pool, wl.num_blocks, wl.page_table.data_ptr(),
                                wl.max_pages, wl.max_pages, wl.start_pos[s].data_ptr(), wl.ones.data_ptr(),
                                wl.B, H, 1, D, BS, _lib.DTYPE_BF16, status, sh)
        _lib.check(rc, "b2pa_kv_append")
        if decode_events is not None:
            decode_events[i][0].record(stream)
        rc = lib.b2pa_paged_decode(wl.q.data_ptr(), s_q, wl.k_pool.data_ptr(), wl.v_pool.data_ptr(), s_pool,
                                   wl.num_blocks, wl.page_table.data_ptr(), wl.max_pages, wl.max_pages,
                                   wl.seq_lens[s].data_ptr(), wl.ones.data_ptr(), wl.out.data_ptr(), s_out,
                                   wl.B, H, D, BS, scale, _lib.DTYPE_BF16, ws.data_ptr(), ws.numel(), status, sh)
        _lib.check(rc, "b2pa_paged_decode")
        if decode_events is not None:
            decode_events[i][1].record(stream)


def count_step_launches(torch, lib, _lib, wl: Workload, dev, step: int, fused: bool = False):
    """Kernels one device step launches, counted from a captured (never
    replayed) CUDA graph of that step: its kernel nodes.  None if the graph
    API is unavailable."""
    try:
        from cuda.bindings import runtime as cudart
    except ImportError:
        return None
    g = torch.cuda.CUDAGraph(keep_graph=True)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        # the capture stream's workspace exists before capture (an allocation
        # inside the graph would add nodes that are not this step's kernels)
        _lib.workspace(dev, lib.b2pa_paged_decode_workspace_size(wl.B, H, D, wl.max_pages, BS, _lib.DTYPE_BF16))
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g, stream=s):
            run_device_steps(torch, lib, _lib, wl, dev, step, 1, fused=fused)
    err, _, n = cudart.cudaGraphGetNodes(g.raw_cuda_graph(), 0)
    if err != cudart.cudaError_t.cudaSuccess:
        return None
    err, nodes, n = cudart.cudaGraphGetNodes(g.raw_cuda_graph(), n)
    kernels = 0
    for node in nodes[:n]:
        err, kind = cudart.cudaGraphNodeGetType(node)
        if err == cudart.cudaError_t.cudaSuccess and kind == cudart.cudaGraphNodeType.cudaGraphNodeTypeKernel:
            kernels += 1
    del g
    return kernels


def build_public_cache(b2pa, wl: Workload, lens_now: np.ndarray):
    """A b2pa BatchedPagedKVCache over the workload's pool, as the allocator
    would have left it at lengths ``lens_now``."""
    pool = b2pa.LayerBlockPool(block_size=BS, initial_blocks=wl.num_blocks, growth_factor=2.0)
    pool.k_blocks, pool.v_blocks = wl.k_pool, wl.v_pool
    pool.num_heads, pool.head_dim, pool.dtype, pool.device = H, D, wl.k_pool.dtype, wl.k_pool.device
    pool.capacity_blocks = wl.num_blocks
    states, in_use = [], set()
    for b in range(wl.B):
        n = int((lens_now[b] + BS - 1) // BS)
        ids = [int(x) for x in wl.table[b, :n]]
        in_use.update(ids)
        states.append(b2pa.PagedKVCacheState(pool=pool, block_ids=ids, seq_len=int(lens_now[b])))
    pool.free_block_ids = [i for i in range(wl.num_blocks) if i not in in_use]
    return b2pa.BatchedPagedKVCache(states, pool=pool)


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons with nvidia-smi every 200 ms in a
    reader thread; ``window`` keeps the samples taken in a time interval."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_id: str):
        import threading

        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", gpu_id], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.perf_counter(), parts))

    def wait_first(self, timeout: float = 5.0) -> None:
        t0 = time.perf_counter()
        while self.proc is not None and not self.samples and time.perf_counter() - t0 < timeout:
            time.sleep(0.05)

    def stop(self, t_from: float, t_to: float) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "samples": 0, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        for ts, parts in self.samples:
            if not (t_from <= ts <= t_to):
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons),
                "window": "pre-load + timed region of the device-resident leg"}


def _gpu_id(local_rank: int) -> str:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local_rank < len(ids):
            return ids[local_rank]
    return str(local_rank)


# ------------------------------------------------------------ CPU baseline
def cpu_baseline(target_seconds: float) -> dict:
    """The CPU restatement of the reference path (oracle/paged_oracle.c) on a
    sample of config[4]: 8 sequences with their own fp32 pool holding the
    same bf16-rounded N(0,1) values, all host threads, repeated until about
    ``target_seconds`` of work; reported as decode tokens/s."""
    from oracle import oracle as orc

    rng = np.random.default_rng(SEED + 77)
    S = 8
    lens = all_lengths(S * 64)[:S]
    pages = ((lens + BS - 1) // BS).astype(np.int64)
    nb = int(pages.sum())
    k = orc.bf16_round(rng.standard_normal((nb, H, BS, D), dtype=np.float32))
    v = orc.bf16_round(rng.standard_normal((nb, H, BS, D), dtype=np.float32))
    q = orc.bf16_round(rng.standard_normal((S, H, 1, D), dtype=np.float32))
    tables, o = [], 0
    for p in pages:
        tables.append(list(range(o, o + int(p))))
        o += int(p)
    threads = orc.c_max_threads()
    t0 = time.perf_counter()
    orc.paged_attention_c(q, k, v, tables, lens.tolist(), [1] * S, nthreads=threads)
    one = time.perf_counter() - t0
    reps = max(1, int(target_seconds / max(one, 1e-3)))
    t0 = time.perf_counter()
    for _ in range(reps):
        orc.paged_attention_c(q, k, v, tables, lens.tolist(), [1] * S, nthreads=threads)
    el = time.perf_counter() - t0
    tok_s = S * reps / el
    th = float(int(lens.sum()) * H * S * reps / el / S)
    return {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{S} config[4] sequences (sum L={int(lens.sum())}), H=32 D=128, bf16 values in fp32, "
                      f"{reps} repetitions, {el:.1f} s; oracle/paged_oracle.c",
            "token_heads_per_s": th * S / S,
            "cpu_model": _cpu_model(), "nproc": os.cpu_count(),
            "reference_torch_loop": reference_loop_rate(min(5.0, target_seconds))}


def reference_loop_rate(target_seconds: float) -> dict:
    """What the reference's own CPU path costs: its loop form
    (oracle/torch_paged.paged_attention_token_loop -- a torch.dot per visible
    token and head, as src/kernels/reference_paged_attention.py:31-57 runs)
    on one config[4] sequence, one head at a time until about
    ``target_seconds``; reported per (token, head) and extrapolated, clearly
    as an estimate, to a full 512-sequence config[4] step."""
    import torch

    from oracle import torch_paged as tp

    lens = all_lengths(512)
    L = int(lens[0])
    n_pages = (L + BS - 1) // BS
    g = torch.Generator().manual_seed(SEED + 78)
    k = torch.randn(n_pages, H, BS, D, generator=g).to(torch.bfloat16).float()
    v = torch.randn(n_pages, H, BS, D, generator=g).to(torch.bfloat16).float()
    q = torch.randn(H, 1, D, generator=g).to(torch.bfloat16).float()
    ids = list(range(n_pages))
    heads = 0
    t0 = time.perf_counter()
    while heads < H and time.perf_counter() - t0 < target_seconds:
        tp.paged_attention_token_loop(q, k, v, ids, L, 1, heads=[heads])
        heads += 1
    el = time.perf_counter() - t0
    rate = L * heads / el
    step_dots = float(lens.sum()) * H
    return {"token_heads_per_s": rate, "seconds": el,
            "sample": f"one config[4] sequence (L={L}), {heads} of {H} heads, fp32 values rounded from bf16",
            "torch_threads": torch.get_num_threads(),
            "estimate_full_step_s": step_dots / rate, "estimate_tok_per_s": 512 * rate / step_dots,
            "estimate": "extrapolated from the per-(token, head) rate to 512 sequences x 32 heads (sum L="
                        f"{int(lens.sum())}); the loop is Python-bound and uses one core"}


def _cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def time_device_leg(torch, lib, _lib, wl: Workload, dev, args, world: int, fused: bool, sample_clocks: bool,
                    local_rank: int = 0):
    """Warm-up, then ``args.steps`` timed steps through the C ABI with inputs
    resident; returns (elapsed ms, per-step decode-call ms, clock record)."""
    import torch.distributed as dist

    run_device_steps(torch, lib, _lib, wl, dev, 0, args.warmup, fused=fused)
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(_gpu_id(local_rank)) if sample_clocks else None
    if clocks is not None:
        clocks.wait_first()
    # Pre-load: repeat the last warm-up step (it rewrites the same row) for
    # ~0.6 s so the clock samples see the GPU under this load (the timed
    # region alone is shorter than the sampling period).
    t_load = time.perf_counter()
    while time.perf_counter() - t_load < 0.6:
        run_device_steps(torch, lib, _lib, wl, dev, args.warmup - 1, 1, fused=fused)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start.record()
    run_device_steps(torch, lib, _lib, wl, dev, args.warmup, args.steps, decode_events=ev, fused=fused)
    end.record()
    torch.cuda.synchronize(dev)
    clock_info = clocks.stop(t_load, time.perf_counter() + 0.25) if clocks is not None else None
    if world > 1:
        dist.barrier()
    status = _lib.read_status(dev)
    if status != 0:
        raise RuntimeError(f"device status {status} after the timed steps")
    return start.elapsed_time(end), [a.elapsed_time(b) for a, b in ev], clock_info


def launch_parity(torch, wl: Workload, step: int, n_random: int = 3) -> dict:
    """Checks the benchmarked launch itself, after the timed region: the
    output of step ``step`` (the last timed one) for a sample of sequences --
    the longest (the most split work items), the shortest, one whose newest
    token opened a fresh block, and ``n_random`` seeded others -- against the
    CPU oracle (oracle/paged_oracle.c) on the same pages, at the bf16
    tolerance (2e-2); and every K/V row the appends wrote into those
    sequences' pages, bit for bit against k_new / v_new."""
    from oracle import oracle as orc

    lens_post = wl.lens0 + step + 1
    picks = [int(np.argmax(lens_post)), int(np.argmin(lens_post))]
    fresh = np.flatnonzero((lens_post - 1) % BS == 0)
    if len(fresh):
        picks.append(int(fresh[0]))
    rng = np.random.default_rng(SEED + 5)
    picks += rng.choice(wl.B, size=min(n_random, wl.B), replace=False).tolist()
    picks = list(dict.fromkeys(picks))
    dev = wl.k_pool.device
    k_pages, v_pages, tables, o = [], [], [], 0
    for b in picks:
        n = int((lens_post[b] + BS - 1) // BS)
        ids = torch.from_numpy(wl.table[b, :n].astype(np.int64)).to(dev)
        k_pages.append(wl.k_pool.index_select(0, ids).cpu())
        v_pages.append(wl.v_pool.index_select(0, ids).cpu())
        tables.append(list(range(o, o + n)))
        o += n
    sel = torch.tensor(picks, device=dev)
    q = wl.q.index_select(0, sel).float().cpu().numpy()
    got = wl.out.index_select(0, sel).float().cpu().numpy()
    ref = orc.paged_attention_c(q, torch.cat(k_pages).float().numpy(), torch.cat(v_pages).float().numpy(), tables,
                                lens_post[picks].tolist(), [1] * len(picks))
    err = np.abs(got - ref)
    out_ok = bool(np.all(err <= 2e-2 + 2e-2 * np.abs(ref)))
    rows_ok, rows = True, 0
    kn = wl.k_new.index_select(0, sel).cpu().view(torch.int16)[:, :, 0]   # [S, H, D]
    vn = wl.v_new.index_select(0, sel).cpu().view(torch.int16)[:, :, 0]
    for i, b in enumerate(picks):
        pos = torch.arange(int(wl.lens0[b]), int(lens_post[b]))
        kr = k_pages[i].view(torch.int16)[pos // BS, :, pos % BS, :]          # [n_appended, H, D]
        vr = v_pages[i].view(torch.int16)[pos // BS, :, pos % BS, :]
        rows += len(pos)
        rows_ok = rows_ok and bool(torch.equal(kr, kn[i].expand_as(kr))) and bool(torch.equal(vr, vn[i].expand_as(vr)))
    return {"seqs": len(picks), "seq_lens": lens_post[picks].tolist(), "max_abs_err": float(err.max()),
            "tolerance": "rtol 2e-2, atol 2e-2 vs oracle/paged_oracle.c", "outputs_ok": out_ok,
            "appended_rows_checked": rows, "appended_rows_bit_exact": rows_ok, "ok": out_ok and rows_ok}


def reduce_parity(torch, parity: dict, dev, world: int) -> dict:
    """Worst case over ranks (every rank calls it, in the same order)."""
    if world == 1:
        return parity
    import torch.distributed as dist

    t = torch.tensor([parity["max_abs_err"], 0.0 if parity["ok"] else 1.0,
                      0.0 if parity["appended_rows_bit_exact"] else 1.0], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    n = torch.tensor([parity["seqs"], parity["appended_rows_checked"]], dtype=torch.int64, device=dev)
    dist.all_reduce(n, op=dist.ReduceOp.SUM)
    return {"seqs": int(n[0]), "ranks": world, "max_abs_err": float(t[0]), "tolerance": parity["tolerance"],
            "appended_rows_checked": int(n[1]), "appended_rows_bit_exact": float(t[2]) == 0.0,
            "ok": float(t[1]) == 0.0}


def e2e_leg(torch, b2pa, wl: Workload, dev, lens_now: np.ndarray, warmup: int, steps: int, fused: bool, world: int):
    """The same step through the public API (BatchedPagedKVCache.append_batch
    + paged_attention) with host buffers: every step uploads its new K, V and
    q (one fused-QKV pinned buffer) and copies its output back to pinned host
    memory, whose arrival the host waits for.  The copies are pipelined as a
    serving loop would: step i+1's upload runs on a copy stream into another
    device buffer while step i decodes, step i's output goes down on another
    copy stream while step i+1 decodes, and the host waits for step i's
    output after it has launched step i+1 (three input buffers, so that a
    step's bulk upload never queues ahead of a step's metadata copy).
    Returns device ms for ``steps``."""
    import torch.distributed as dist

    cache = build_public_cache(b2pa, wl, lens_now)
    B = wl.B
    comp = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    d2h_stream = torch.cuda.Stream(dev)
    host_kvq = torch.randn(B, 1, 3, H, D, dtype=torch.bfloat16).pin_memory()
    host_out = [torch.empty(B, H, 1, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    # three input buffers: step i+2's upload goes into step i-1's buffer and
    # is enqueued once step i-1's output has arrived -- after step i's small
    # metadata copy on the compute stream, which would otherwise wait behind
    # the bulk copy in the host-to-device copy engine
    NBUF = 3
    dev_kvq = [torch.empty(B, 1, 3, H, D, dtype=torch.bfloat16, device=dev) for _ in range(NBUF)]
    up_ev = [torch.cuda.Event() for _ in range(NBUF)]
    free_ev = [torch.cuda.Event() for _ in range(NBUF)]
    out_ev = [torch.cuda.Event() for _ in range(2)]
    for e in free_ev:
        e.record(comp)

    def upload(i):
        j = i % NBUF
        copy_stream.wait_event(free_ev[j])          # step i-3 is done reading this buffer
        with torch.cuda.stream(copy_stream):
            dev_kvq[j].copy_(host_kvq, non_blocking=True)
        up_ev[j].record(copy_stream)

    def compute(i):
        j, o = i % NBUF, i % 2
        comp.wait_event(up_ev[j])
        k, v, q = (dev_kvq[j][:, :, c].transpose(1, 2) for c in range(3))
        cache.append_batch(k, v, 1)
        out = b2pa.paged_attention("b200_paged", q, cache, 1)
        free_ev[j].record(comp)                     # also: this step's output is written
        d2h_stream.wait_event(free_ev[j])
        out.record_stream(d2h_stream)
        with torch.cuda.stream(d2h_stream):
            host_out[o].copy_(out, non_blocking=True)
        out_ev[o].record(d2h_stream)

    def run(n):
        copy_stream.wait_stream(comp)
        for i in range(min(2, n)):
            upload(i)
        for i in range(n):
            compute(i)
            if i >= 1:
                out_ev[(i - 1) % 2].synchronize()      # step i-1's output is on the host
            # enqueued only now, behind step i's metadata copy in the copy
            # engine; it runs while step i decodes
            if i + 2 < n:
                upload(i + 2)
        out_ev[(n - 1) % 2].synchronize()

    fused_before = b2pa.set_fused_append(fused)
    try:
        run(warmup)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(comp)
        run(steps)
        comp.wait_stream(d2h_stream)
        e_end.record(comp)
        torch.cuda.synchronize(dev)
    finally:
        b2pa.set_fused_append(fused_before)
    from b2pa import _lib

    _lib.raise_on_device_status(dev, "e2e steps")
    return e_start.elapsed_time(e_end)


# --------------------------------------------------------------------- main
def main(argv=None) -> int:
    args = parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return main_reference(args, rank, world)
    if args.workload != "decode":
        return main_secondary(args)

    import torch
    import torch.distributed as dist

    import b2pa
    from b2pa import _lib

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.load()
    e2e_steps = args.e2e_steps or args.steps
    total_steps = args.warmup + args.steps + args.warmup + e2e_steps + 1
    lens0 = my_sequences(args, rank, world)
    wl = Workload(torch, dev, lens0, total_steps, rank)
    torch.cuda.synchronize(dev)

    # ---------------------------------------------- device-resident (value)
    fused = args.decode_append == "fused"
    run_device_steps(torch, lib, _lib, wl, dev, 0, args.warmup, fused=fused)
    torch.cuda.synchronize(dev)
    launches_per_step = count_step_launches(torch, lib, _lib, wl, dev, args.warmup, fused=fused)
    elapsed_ms, decode_ms, clock_info = time_device_leg(torch, lib, _lib, wl, dev, args, world, fused, True,
                                                        local_rank)
    # parity of the benchmarked launch: the last timed step's output and the rows the appends wrote
    parity = reduce_parity(torch, launch_parity(torch, wl, args.warmup + args.steps - 1), dev, world)

    # --------------------------------------------------- end to end (e2e)
    lens_now = wl.lens0 + args.warmup + args.steps
    e2e_ms = e2e_leg(torch, b2pa, wl, dev, lens_now, args.warmup, e2e_steps, fused, world)
    B = wl.B
    pool_gb = wl.pool_bytes() / 1e9
    sum_len = int(wl.lens0.sum())

    # ------------------------------------------------------ aggregate
    elapsed_ms, e2e_ms, decode_avg_ms = max_over_ranks([elapsed_ms, e2e_ms, float(np.mean(decode_ms))], dev, world)
    total_seqs = B * world
    value = total_seqs * args.steps / (elapsed_ms / 1e3)
    e2e_value = total_seqs * e2e_steps / (e2e_ms / 1e3)

    # roofline of the dominant kernel (decode), per launch, averaged over the timed steps
    lens_timed = [wl.lens0 + args.warmup + i + 1 for i in range(args.steps)]
    bytes_per_launch = float(np.mean([algorithmic_decode_bytes(x) for x in lens_timed]))
    if fused:  # the fused launch also reads the new K/V rows and writes them to the pool
        bytes_per_launch += 4 * B * H * D * 2
    del wl
    torch.cuda.empty_cache()

    # --------------------------------------------- strong scaling (same run)
    # The fixed BASELINE config[4] draw of ``--seqs`` sequences spread over the
    # ranks; at N=1 it is the workload above.
    strong = None
    if world > 1 and args.scaling == "weak":
        swl = Workload(torch, dev, my_sequences(args, rank, world, "strong"), total_steps, rank)
        s_ms, s_dec, _ = time_device_leg(torch, lib, _lib, swl, dev, args, world, fused, False, local_rank)
        s_parity = reduce_parity(torch, launch_parity(torch, swl, args.warmup + args.steps - 1), dev, world)
        s_ms, s_dec_avg = max_over_ranks([s_ms, float(np.mean(s_dec))], dev, world)
        strong = {"value": args.seqs * args.steps / (s_ms / 1e3), "unit": "tok/s",
                  "ms_per_step": s_ms / args.steps, "decode_ms_per_launch": s_dec_avg,
                  "sequences_total": args.seqs, "sequences_per_gpu": swl.B, "parity": s_parity}
        del swl
        torch.cuda.empty_cache()
    elif world == 1:
        strong = {"value": value, "unit": "tok/s", "ms_per_step": elapsed_ms / args.steps,
                  "decode_ms_per_launch": decode_avg_ms, "sequences_total": B, "sequences_per_gpu": B,
                  "note": "one GPU: the strong-scaling workload is the workload of this line"}

    peaks = _peaks()
    achieved_gbs = bytes_per_launch / (decode_avg_ms / 1e3) / 1e9
    result = {
        "metric": "paged_decode_tokens_per_s",
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) bf16 K/V pools, queries and new tokens; seeded U[1024,8192] lengths",
        "config": {
            "workload": "BASELINE config[4] large paged decode: per step one 1-token KV append + one decode "
                        "per sequence; H=32, D=128, bf16, block 16, L~U[1024,8192], pool 1.2x pages",
            "decode_append": ("fused: one b2pa_paged_decode_append per step" if fused else
                              "separate: b2pa_kv_append + b2pa_paged_decode per step"),
            "sequences_per_gpu": B,
            "sequences_total": total_seqs,
            "sum_len_rank0": sum_len,
            "partition": "token-balanced: longest first to the rank with the fewest tokens, equal counts",
            "pool_gb_per_gpu": pool_gb,
            "parallelism": f"sequence-partitioned dp{world}, one pool per rank, no hot-path collective",
            "l2": "inputs larger than L2 (K/V pool of tens of GB per GPU); no flush needed",
            **({"len_range": "U[%d,%d], not config[4]'s" % tuple(args.len_range)} if args.len_range else {}),
        },
        "hbm_gb_per_s_decode": achieved_gbs,
        "roofline": {
            "bound": "hbm",
            "kernel": ("paged_decode with the fused append (every launch of one b2pa_paged_decode_append call: the "
                       "decode kernel and, when a sequence is split, the combine)" if fused else
                       "paged_decode (every launch of one b2pa_paged_decode call: the decode kernel and, when a "
                       "sequence is split, the combine)"),
            "achieved": achieved_gbs,
            "peak": peaks["hbm_gbs"],
            "peak_source": peaks["source"],
            "unit": "GB/s",
            "frac": achieved_gbs / peaks["hbm_gbs"],
            "frac_of_nominal_8tbs": achieved_gbs / 8000.0,
            "algorithmic_bytes_per_launch": bytes_per_launch,
            "decode_ms_per_launch": decode_avg_ms,
            # DRAM bytes per launch: the ncu capture of this kernel on the
            # 16-sequence case (1.4386 GB read + 6.6 MB written for 1.4373 GB
            # algorithmic) scaled to this launch by its algorithmic bytes; its
            # long contexts have config[4]'s share of partial last pages (a
            # 300-sequence capture of the contiguous split read the
            # algorithmic bytes plus its page tails within 0.03 %)
            "traffic": bytes_per_launch * DECODE_TRAFFIC_PER_ALGORITHMIC_BYTE,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the 16-sequence capture, "
                              "scaled by algorithmic bytes",
        },
        "parity": parity,
        "e2e": {
            "value": e2e_value,
            "unit": "tok/s",
            "ms_per_step": e2e_ms / e2e_steps,
            "h2d_bytes_per_step": 3 * B * H * D * 2,
            "d2h_bytes_per_step": B * H * D * 2,
            "path": "b2pa.BatchedPagedKVCache.append_batch + b2pa.paged_attention, pinned host inputs and outputs, "
                    "uploads on a copy stream one step ahead, outputs down on another copy stream and awaited "
                    "after the next step's launch"
                    + (", b2pa.set_fused_append(True)" if fused else ""),
        },
        "strong": strong,
        "gpu_launches": (launches_per_step * args.steps) if launches_per_step is not None else None,
        "gpu_launches_per_step": launches_per_step,
        "clocks": clock_info,
    }
    if rank == 0 and world == 1 and not args.no_secondary:
        result["secondary"] = secondary_summary(args)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result))
    ok = parity["ok"] and (strong is None or strong.get("parity", {"ok": True})["ok"])
    if not ok:
        print("bench: the benchmarked launch does not match the oracle", file=sys.stderr)
        return 1
    return 0


# ------------------------------------------------------ secondary workloads
def _prefill_flops(prefix: np.ndarray, T: int, H: int, D: int) -> float:
    """4*H*D flops per (query row, visible key): row t of a chunk over a
    prefix P sees P + t + 1 keys."""
    return float(4 * H * D * np.sum(T * prefix + T * (T + 1) // 2))


def _secondary_case(workload: str, prefix_len: int | None = None):
    """Inputs of BASELINE config[2] (``prefill``: B=8 chunks of 256 tokens over
    prefixes U[0,768], or every prefix ``prefix_len``) or config[1]
    (``decode_f32``: 64 sequences, context U[128,1024] before the step's
    token); H=8, D=64, block 16, random tables over a 4096-block pool."""
    rng = np.random.default_rng(2 if workload == "prefill" else 1)
    B = 8 if workload == "prefill" else 64
    T = 256 if workload == "prefill" else 1
    if workload == "prefill":
        prefix = rng.integers(0, 769, size=B)
        if prefix_len is not None:
            prefix = np.full(B, prefix_len, dtype=np.int64)
    else:
        prefix = rng.integers(128, 1025, size=B)  # context before this step's token
    return rng, B, T, prefix


def measure_secondary(torch, lib, _lib, dev, workload: str, dtype, steps: int, warmup: int,
                      cpu_seconds: float | None = None, prefix_len: int | None = None) -> dict:
    """Kernel-level measurement of one secondary case through the C ABI with
    device-resident inputs: the append + attention step (eager, L2 flushed),
    the same step as one fused call, and the attention alone as a CUDA-graph
    replay (device time without host launch gaps)."""
    status = _lib.status_buffer(dev).data_ptr()
    peaks = _peaks()
    Hs, Ds, NB, bs = 8, 64, 4096, 16
    rng, B, T, prefix = _secondary_case(workload, prefix_len)
    lens = prefix + T
    pages = (lens + bs - 1) // bs
    perm = rng.permutation(NB).astype(np.int32)
    max_pages = int(pages.max())
    table = np.full((B, max_pages), -1, dtype=np.int32)
    o = 0
    for b in range(B):
        table[b, :pages[b]] = perm[o:o + pages[b]]
        o += int(pages[b])
    gen = torch.Generator(device=dev).manual_seed(7)
    kp = torch.randn(NB, Hs, bs, Ds, generator=gen, device=dev).to(dtype)
    vp = torch.randn_like(kp)
    x = torch.randn(B, T, 3, Hs, Ds, generator=gen, device=dev).to(dtype)
    kn, vn, q = (x[:, :, i].transpose(1, 2) for i in range(3))
    out = torch.empty_like(q)
    pt = torch.from_numpy(table).to(dev)
    start = torch.from_numpy(prefix.astype(np.int32)).to(dev)
    seq = torch.from_numpy(lens.astype(np.int32)).to(dev)
    cur = torch.full((B,), T, dtype=torch.int32, device=dev)
    dt = _lib.dtype_code(dtype)
    sh = torch.cuda.current_stream(dev).cuda_stream
    scale = 1.0 / math.sqrt(Ds)
    ws_n = (lib.b2pa_paged_decode_workspace_size(B, Hs, Ds, max_pages, bs, dt) if T == 1 else
            lib.b2pa_paged_prefill_workspace_size(B, Hs, T, Ds, max_pages, bs, dt))
    ws = _lib.workspace(dev, max(ws_n, 1))

    def append():
        _lib.check(lib.b2pa_kv_append(kn.data_ptr(), _lib.strides4(kn), vn.data_ptr(), _lib.strides4(vn),
                                      kp.data_ptr(), vp.data_ptr(), _lib.strides4(kp), NB, pt.data_ptr(),
                                      max_pages, max_pages, start.data_ptr(), cur.data_ptr(), B, Hs, T, Ds,
                                      bs, dt, status, sh), "append")

    def attend():
        if T == 1:
            rc = lib.b2pa_paged_decode(q.data_ptr(), _lib.strides4(q), kp.data_ptr(), vp.data_ptr(),
                                       _lib.strides4(kp), NB, pt.data_ptr(), max_pages, max_pages,
                                       seq.data_ptr(), cur.data_ptr(), out.data_ptr(), _lib.strides4(out),
                                       B, Hs, Ds, bs, scale, dt, ws.data_ptr(), ws.numel(), status, sh)
        else:
            rc = lib.b2pa_paged_prefill(q.data_ptr(), _lib.strides4(q), kp.data_ptr(), vp.data_ptr(),
                                        _lib.strides4(kp), NB, pt.data_ptr(), max_pages, max_pages,
                                        seq.data_ptr(), cur.data_ptr(), out.data_ptr(), _lib.strides4(out),
                                        B, Hs, T, Ds, bs, scale, dt, ws.data_ptr(), ws.numel(), status, sh)
        _lib.check(rc, "attention")

    for _ in range(max(warmup, 3)):
        append()
        attend()
    torch.cuda.synchronize()
    # L2 flush (the config[2]/[1] working sets fit in the 126 MB L2): write
    # a 256 MB buffer, then read another one, so the timed kernels start
    # on an L2 holding only clean, unrelated lines (no write-backs of the
    # flush's dirty lines inside the timed region).
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_r = torch.zeros(32 << 20, dtype=torch.int64, device=dev)

    class _Flush:
        @staticmethod
        def zero_():
            flush_w.zero_()
            flush_r.sum()

    flush = _Flush()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1, e2 in ev:
        flush.zero_()
        e0.record()
        append()
        e1.record()
        attend()
        e2.record()
    torch.cuda.synchronize()
    _lib.raise_on_device_status(dev, "secondary bench")
    step_ms = float(np.mean([a.elapsed_time(c) for a, _, c in ev]))
    # the same step as one call: b2pa_paged_decode_append (T == 1) or
    # b2pa_paged_prefill_append (the chunk's append inside the fp32
    # tensor-core path's page copy; append kernel + prefill otherwise)
    def fused():
        if T == 1:
            _lib.check(lib.b2pa_paged_decode_append(
                q.data_ptr(), _lib.strides4(q), kn.data_ptr(), _lib.strides4(kn), vn.data_ptr(),
                _lib.strides4(vn), kp.data_ptr(), vp.data_ptr(), _lib.strides4(kp), NB, pt.data_ptr(),
                max_pages, max_pages, seq.data_ptr(), cur.data_ptr(), start.data_ptr(), cur.data_ptr(), None,
                out.data_ptr(), _lib.strides4(out), B, Hs, Ds, bs, scale, dt, ws.data_ptr(), ws.numel(),
                status, sh), "decode_append")
        else:
            _lib.check(lib.b2pa_paged_prefill_append(
                q.data_ptr(), _lib.strides4(q), kn.data_ptr(), _lib.strides4(kn), vn.data_ptr(),
                _lib.strides4(vn), kp.data_ptr(), vp.data_ptr(), _lib.strides4(kp), NB, pt.data_ptr(),
                max_pages, max_pages, seq.data_ptr(), cur.data_ptr(), start.data_ptr(), cur.data_ptr(), None,
                out.data_ptr(), _lib.strides4(out), B, Hs, T, Ds, bs, scale, dt, ws.data_ptr(), ws.numel(),
                status, sh), "prefill_append")

    for _ in range(max(warmup, 3)):
        fused()
    fev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in fev:
        flush.zero_()
        e0.record()
        fused()
        e1.record()
    torch.cuda.synchronize()
    _lib.raise_on_device_status(dev, "secondary bench (fused)")
    fused_ms = float(np.mean([a.elapsed_time(b) for a, b in fev]))
    attn_eager_ms = float(np.mean([b.elapsed_time(c) for _, b, c in ev]))
    # Device time without host launch gaps: the attention call captured in
    # a CUDA graph and replayed (L2 flushed before every replay).
    g = torch.cuda.CUDAGraph()
    s_cap = torch.cuda.Stream()
    s_cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s_cap):
        sh = s_cap.cuda_stream
        attend()
        with torch.cuda.graph(g, stream=s_cap):
            attend()
    torch.cuda.current_stream().wait_stream(s_cap)
    sh = torch.cuda.current_stream(dev).cuda_stream
    gev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in gev:
        flush.zero_()
        e0.record()
        g.replay()
        e1.record()
    torch.cuda.synchronize()
    attn_ms = float(np.mean([a.elapsed_time(b) for a, b in gev]))
    del g
    # Per-call device time without the graph launch and event overhead of a
    # single replay (~6 us on this part even for a trivial kernel): a graph of
    # 10 x (L2 flush, attention call) minus a graph of the 10 flushes alone.
    def graph_of(n, with_attention):
        gg = torch.cuda.CUDAGraph()
        s2 = torch.cuda.Stream()
        s2.wait_stream(torch.cuda.current_stream())
        nonlocal sh
        with torch.cuda.stream(s2):
            sh = s2.cuda_stream
            with torch.cuda.graph(gg, stream=s2):
                for _ in range(n):
                    flush.zero_()
                    if with_attention:
                        attend()
        torch.cuda.current_stream().wait_stream(s2)
        sh = torch.cuda.current_stream(dev).cuda_stream
        return gg

    def replay_ms(gg, reps=5):
        ts = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            gg.replay()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return float(np.median(ts))

    g_both, g_flush = graph_of(10, True), graph_of(10, False)
    attn_in_graph_ms = (replay_ms(g_both) - replay_ms(g_flush)) / 10
    del g_both, g_flush
    es = 2 if dtype == torch.bfloat16 else 4
    kv_bytes = 2 * Hs * Ds * es * int(lens.sum())
    line = {"workload": workload, "dtype": str(dtype).replace("torch.", ""), "steps": steps,
            "config": {"B": B, "H": Hs, "D": Ds, "T": T, "block_size": bs, "pool_blocks": NB,
                       "l2": "flushed before every step (256 MB written, then 256 MB read)"},
            "ms_per_step_append_plus_attention": step_ms, "attention_ms": attn_ms,
            "attention_ms_in_graph": attn_in_graph_ms,
            "attention_ms_eager_call": attn_eager_ms, "append_ms": step_ms - attn_eager_ms,
            "timing": "attention_ms: one CUDA-graph replay of the call between two events (device time, incl. the "
                      "replay's launch overhead); attention_ms_in_graph: per call inside a graph of 10 flushed "
                      "calls, minus the flushes; eager: per-call incl. host launch"}
    if T > 1:
        flops = _prefill_flops(prefix, T, Hs, Ds)
        bytes_ = kv_bytes + 2 * B * Hs * T * Ds * es
        line.update({"tokens_per_s": B * T / (step_ms / 1e3),
                     "ms_per_step_fused_append_prefill": fused_ms,
                     "tokens_per_s_fused": B * T / (fused_ms / 1e3),
                     "attention_tflops": flops / (attn_ms / 1e3) / 1e12,
                     "attention_tflops_in_graph": flops / (attn_in_graph_ms / 1e3) / 1e12,
                     "frac_of_bf16_tensor_peak_in_graph": flops / (attn_in_graph_ms / 1e3) / 1e12
                     / peaks["bf16_tflops"],
                     "flops_per_launch": flops, "bytes_per_launch": bytes_,
                     "attention_hbm_gbs": bytes_ / (attn_ms / 1e3) / 1e9,
                     "frac_of_bf16_tensor_peak": flops / (attn_ms / 1e3) / 1e12 / peaks["bf16_tflops"],
                     "frac_of_hbm_peak": bytes_ / (attn_ms / 1e3) / 1e9 / peaks["hbm_gbs"]})
    else:
        bytes_ = kv_bytes + 2 * B * Hs * Ds * es + 4 * int(pages.sum()) + 8 * B
        line.update({"tokens_per_s": B / (step_ms / 1e3),
                     "ms_per_step_fused_append_decode": fused_ms,
                     "tokens_per_s_fused": B / (fused_ms / 1e3),
                     "attention_hbm_gbs": bytes_ / (attn_ms / 1e3) / 1e9,
                     "attention_hbm_gbs_in_graph": bytes_ / (attn_in_graph_ms / 1e3) / 1e9,
                     "bytes_per_launch": bytes_,
                     "frac_of_hbm_peak": bytes_ / (attn_ms / 1e3) / 1e9 / peaks["hbm_gbs"]})
    if cpu_seconds is not None:
        line["cpu_baseline"] = _secondary_cpu_baseline(kp, vp, q, table, pages, lens, T, cpu_seconds)
    del kp, vp, flush
    torch.cuda.empty_cache()
    return line




def main_secondary(args) -> int:
    """Kernel-level measurements of BASELINE config[2] (chunked prefill, bf16
    and fp32) and config[1] (fp32 decode + append); one JSON line per dtype."""
    import torch

    from b2pa import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    dtypes = [torch.bfloat16, torch.float32] if args.workload == "prefill" else [torch.float32]
    for dtype in dtypes:
        line = measure_secondary(torch, lib, _lib, dev, args.workload, dtype, args.steps, args.warmup,
                                 None if args.no_cpu_baseline else args.cpu_seconds)
        print(json.dumps(line))
    return 0


def measure_decode_step(torch, dev, steps: int = 120, prompt: int = 128) -> dict:
    """config[0]'s decode step on b2pa kernels: b2pa.FusedDecoder (row kernels +
    the fused append/decode) replayed as a CUDA graph (b2pa.DecodeGraph), batch
    1, after a 128-token prompt.  The weights are seeded random values in a
    parameter container with the config[0] model's shapes under the
    reference's module names (vocab 5000, d_model 512, 8 heads, 6 layers,
    d_ff 2048); the prompt's K/V rows are random, appended to every layer's
    pool through BatchedPagedKVCache.append_batch.  Tokens stay on the device;
    one synchronisation at the end.  (Correctness of this path is checked by
    the GPU tests against the reference's tokens.)"""
    import torch.nn as nn

    import b2pa

    V, d, Hh, L, dff = 5000, 512, 8, 6, 2048

    class _Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.num_heads = Hh
            self.q_proj, self.k_proj, self.v_proj, self.out_proj = (nn.Linear(d, d) for _ in range(4))

    class _Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.ln1, self.attn, self.ln2 = nn.LayerNorm(d), _Attn(), nn.LayerNorm(d)
            self.mlp = nn.Sequential(nn.Linear(d, dff), nn.GELU(), nn.Linear(dff, d))

    class _Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.token_emb, self.pos_emb = nn.Embedding(V, d), nn.Embedding(1024, d)
            self.blocks = nn.ModuleList(_Block() for _ in range(L))
            self.ln_f, self.lm_head = nn.LayerNorm(d), nn.Linear(d, V, bias=False)

    torch.manual_seed(SEED)
    model = _Model().to(dev).eval()
    gen = torch.Generator(device=dev).manual_seed(SEED)
    states = []
    for _ in range(L):
        pool = b2pa.LayerBlockPool(block_size=16, initial_blocks=64, growth_factor=2.0)
        st = b2pa.PagedKVCacheState(pool=pool)
        kv = torch.randn(2, 1, Hh, prompt, d // Hh, generator=gen, device=dev)
        b2pa.BatchedPagedKVCache([st], pool=pool).append_batch(kv[0], kv[1], prompt)
        states.append(st)
    layer_states = [[st] for st in states]
    batches = [b2pa.BatchedPagedKVCache([st], pool=st.pool) for st in states]
    dec = b2pa.FusedDecoder(model, max_batch=1)
    ids = torch.zeros(1, dtype=torch.int64, device=dev)
    pos = torch.zeros(1, dtype=torch.int64, device=dev)
    toks = torch.empty(steps, dtype=torch.int64, device=dev)
    graph = b2pa.DecodeGraph(lambda: dec.step(ids, pos, batches)[1])
    with torch.no_grad():
        for s in range(3):  # warm-up and capture
            pos.fill_(prompt + s)
            ids.copy_(graph(layer_states))
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for s in range(steps):
            pos.fill_(prompt + 3 + s)
            nx = graph(layer_states)
            toks[s] = nx[0]
            ids.copy_(nx)
        torch.cuda.synchronize(dev)
        secs = time.perf_counter() - t0
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(20):  # replays rewrite the last step's rows with the same values
            graph.graph.replay()
        b.record()
        torch.cuda.synchronize(dev)
    weights = sum(p.numel() for n, p in model.named_parameters() if "emb" not in n) * 4
    return {"tokens_per_s": steps / secs, "ms_per_token": secs / steps * 1e3,
            "device_us_per_step": a.elapsed_time(b) / 20 * 1e3, "graph_captures": graph.captures,
            "weight_bytes_per_step": weights,
            "what": "config[0] decode step (batch 1, 128-token prompt, 6 layers, fp32) on b2pa.FusedDecoder as a "
                    "CUDA graph; seeded random weights with the config[0] shapes"}


def secondary_summary(args) -> dict:
    """The secondary kernels timed inside the main bench run (one GPU):
    config[2] chunked prefill bf16 and fp32, the same with 4096-token
    prefixes, and config[1] fp32 decode + append."""
    import torch

    from b2pa import _lib

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    keep = ("attention_ms", "attention_ms_in_graph", "attention_tflops", "attention_tflops_in_graph",
            "frac_of_bf16_tensor_peak", "frac_of_bf16_tensor_peak_in_graph", "attention_hbm_gbs_in_graph",
            "frac_of_hbm_peak",
            "attention_hbm_gbs", "ms_per_step_append_plus_attention", "ms_per_step_fused_append_prefill",
            "ms_per_step_fused_append_decode", "tokens_per_s_fused")
    out = {}
    cases = [("prefill_bf16_config2", "prefill", torch.bfloat16, None),
             ("prefill_f32_config2", "prefill", torch.float32, None),
             ("prefill_bf16_prefix4096", "prefill", torch.bfloat16, 4096),
             ("prefill_f32_prefix4096", "prefill", torch.float32, 4096),
             ("decode_append_f32_config1", "decode_f32", torch.float32, None)]
    for name, workload, dtype, plen in cases:
        line = measure_secondary(torch, lib, _lib, dev, workload, dtype, max(args.steps, 10), args.warmup,
                                 None, plen)
        out[name] = {k: line[k] for k in keep if k in line}
    out["decode_step_config0"] = measure_decode_step(torch, dev)
    out["timing"] = ("CUDA events; L2 flushed before every call; attention_ms: one CUDA-graph replay of the call "
                     "(includes ~6 us of replay launch overhead); attention_ms_in_graph: per call inside a graph of "
                     "10 flushed calls minus the flushes; step times: eager calls")
    return out


def _secondary_cpu_baseline(kp, vp, q, table, pages, lens, T, target_seconds: float) -> dict:
    """The CPU restatement of the reference's torch path (oracle/paged_oracle.c,
    all host threads) on the same inputs, repeated to about target_seconds."""
    from oracle import oracle as orc

    k_h = kp.float().cpu().numpy()
    v_h = vp.float().cpu().numpy()
    q_h = q.float().cpu().numpy()
    tables = [[int(x) for x in table[b, :pages[b]]] for b in range(len(lens))]
    cur = [T] * len(lens)
    threads = orc.c_max_threads()
    t0 = time.perf_counter()
    orc.paged_attention_c(q_h, k_h, v_h, tables, lens.tolist(), cur, nthreads=threads)
    one = time.perf_counter() - t0
    reps = max(1, int(target_seconds / max(one, 1e-3)))
    t0 = time.perf_counter()
    for _ in range(reps):
        orc.paged_attention_c(q_h, k_h, v_h, tables, lens.tolist(), cur, nthreads=threads)
    sec = (time.perf_counter() - t0) / reps
    return {"value": len(lens) * T / sec, "unit": "tok/s", "seconds_per_step": sec, "cores": threads,
            "kind": "port", "sample": f"full step, {reps} repetitions; attention only (oracle/paged_oracle.c)",
            "cpu_model": _cpu_model()}


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def main_reference(args, rank: int, world: int) -> int:
    """Reference arm: the CPU restatement of the reference's torch path."""
    if rank != 0:
        return 0
    from oracle import oracle as orc

    orc.build_c_oracle()
    rng = np.random.default_rng(SEED + 99)
    S = 32
    lens = all_lengths(S * 64)[:S]
    pages = ((lens + BS - 1) // BS).astype(np.int64)
    nb = int(pages.sum())
    k = orc.bf16_round(rng.standard_normal((nb, H, BS, D), dtype=np.float32))
    v = orc.bf16_round(rng.standard_normal((nb, H, BS, D), dtype=np.float32))
    q = orc.bf16_round(rng.standard_normal((S, H, 1, D), dtype=np.float32))
    tables, o = [], 0
    for p in pages:
        tables.append(list(range(o, o + int(p))))
        o += int(p)
    threads = orc.c_max_threads()
    for _ in range(args.warmup):
        orc.paged_attention_c(q, k, v, tables, lens.tolist(), [1] * S, nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.paged_attention_c(q, k, v, tables, lens.tolist(), [1] * S, nthreads=threads)
    el = time.perf_counter() - t0
    value = S * args.steps / el
    sample = (f"each step: {S} config[4] sequences (sum L={int(lens.sum())}), H=32 D=128, bf16 values in fp32, "
              f"oracle/paged_oracle.c (restatement of src/kernels/reference_paged_attention.py)")
    print(json.dumps({
        "impl": "reference",
        "metric": "paged_decode_tokens_per_s",
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": el * 1e3 / args.steps,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded N(0,1) values rounded to bf16; seeded U[1024,8192] lengths",
        "config": {"workload": f"BASELINE config[4] large paged decode (CPU sample of {S} sequences per step)",
                   "sequences_per_step": S},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample,
                         "cpu_model": _cpu_model(), "nproc": os.cpu_count()},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))
    return 0


if __name__ == "__main__":
    sys.exit(main())
