"""A decode step planned once for every layer, and the step as a CUDA graph.

In the reference every layer's forward repeats the same host work for a
decode step: ``append_batch`` allocates the layer's blocks and copies the
new K/V row (src/cache/paged_kv.py:151-172), then ``paged_attention`` builds
the block table and lengths from Python lists and copies them to the device
(src/cache/paged_kv.py:174-197, src/kernels/paged_attention.py:25-26), and
the generation loop re-stacks the request caches per layer every step
(src/inference/generate_with_cache.py:48-67).  Allocation is lockstep: every
layer's pool sees the same requests in the same order, so every layer hands
out the same block ids.  Here that is checked, not assumed, and used:

* ``DecodeStep.begin`` allocates the step's token for every request in every
  layer (each layer's own pool, in the reference's batch order), checks that
  all layers now hold identical block tables, and uploads ONE block table and
  one set of lengths/positions, shared by all layers, into device buffers
  whose addresses stay fixed from step to step;
* while the step is open, ``append_batch`` on those caches does no host work
  (it leaves the row copy to the attention call) and ``paged_attention``
  launches ``b2pa_paged_decode_append`` on the shared buffers: one launch per
  layer, no allocation, no upload, no host synchronisation;
* ``DecodeGraph`` captures a caller's decode-step function (the model's
  forward for one token, with its embeddings, projections, MLP, lm_head and
  sampling) in a CUDA graph once and replays it every step: per step the host
  only allocates blocks and uploads the shared metadata (and the caller's
  inputs).  A change that moves a buffer the graph has baked in -- a pool that
  grew (``torch.cat`` moves it), a table that outgrew its width, a different
  batch -- makes the next step capture again.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._staging import _cudart, _rt_check


class SharedStepMetadata:
    """Device buffers every layer's decode launch reads, at fixed addresses:
    int32 ``[table (capacity x width) | seq_lens | start_pos | ones]`` (each
    row segment ``capacity`` long) and the int64 lengths ``append_batch``
    returns.  A step of B <= capacity requests uses the first B rows of each."""

    RING = 4  # pinned host copies: the host may plan this many steps ahead of the GPU

    def __init__(self, device: torch.device, B: int, width: int):
        self.device, self.B, self.width = device, B, width
        self.capacity = B
        n = B * width + 3 * B
        self.dev = torch.empty(n, dtype=torch.int32, device=device)
        self.hosts = [torch.empty(n, dtype=torch.int32, pin_memory=True) for _ in range(self.RING)]
        for h in self.hosts:
            h.numpy()[B * width + 2 * B:] = 1
        rt = _cudart()
        self.events = []
        with torch.cuda.device(device):
            for _ in range(self.RING):
                ev = ctypes.c_void_p()
                _rt_check(rt.cudaEventCreateWithFlags(ctypes.byref(ev), 2), "cudaEventCreateWithFlags")
                self.events.append(ev)
        self.recorded = [False] * self.RING
        self.slot = 0
        self.nbytes = 4 * n
        self.seq_out = torch.empty(B, dtype=torch.int64, device=device)
        self.workspace: torch.Tensor | None = None
        self._ws_key = None

    def __del__(self):
        # the ring's events; the CUDA runtime may already be gone at exit
        try:
            rt = _cudart()
            for ev in getattr(self, "events", []):
                rt.cudaEventDestroy(ev)
        except Exception:  # noqa: BLE001 -- nothing to clean up with then
            pass

    @property
    def table(self) -> torch.Tensor:
        return self.dev[: self.capacity * self.width]

    def _row(self, i: int) -> torch.Tensor:
        o = self.capacity * self.width + i * self.capacity
        return self.dev[o: o + self.capacity]

    @property
    def seq_lens(self) -> torch.Tensor:
        return self._row(0)

    @property
    def start_pos(self) -> torch.Tensor:
        return self._row(1)

    @property
    def ones(self) -> torch.Tensor:
        return self._row(2)

    def upload(self, tables: list, seq_lens: list[int], starts: list[int]) -> None:
        """Writes the step's table and rows; one copy on the current stream,
        from the next pinned buffer of a small ring (rewritten only once the
        copy that last read it is done, so the host can plan a few steps ahead
        of the GPU without waiting)."""
        i = self.slot
        self.slot = (i + 1) % self.RING
        rt = _cudart()
        if self.recorded[i]:
            _rt_check(rt.cudaEventSynchronize(self.events[i]), "cudaEventSynchronize")
        host = self.hosts[i]
        h = host.numpy()
        C, W, B = self.capacity, self.width, len(tables)
        t = h[: B * W].reshape(B, W)
        t.fill(-1)
        for r, ids in enumerate(tables):
            if ids:
                t[r, : len(ids)] = ids
        h[C * W: C * W + B] = seq_lens
        h[C * W + C: C * W + C + B] = starts
        stream = _lib.stream_handle(self.device)
        _rt_check(rt.cudaMemcpyAsync(self.dev.data_ptr(), host.data_ptr(), self.nbytes, 1, stream), "cudaMemcpyAsync")
        _rt_check(rt.cudaEventRecord(self.events[i], stream), "cudaEventRecord")
        self.recorded[i] = True

    def ensure_workspace(self, H: int, D: int, block_size: int, dtype: torch.dtype) -> torch.Tensor:
        key = (H, D, block_size, dtype)
        if key == self._ws_key:
            return self.workspace
        self._ws_key = key
        lib = _lib.load()
        # enough for every batch size the buffers serve (the split plan is not
        # monotone in B)
        need = max(lib.b2pa_paged_decode_workspace_size(b, H, D, self.width, block_size, _lib.dtype_code(dtype))
                   for b in range(1, self.capacity + 1))
        if self.workspace is None or self.workspace.numel() < need:
            self.workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
        return self.workspace


class _StepPending:
    """The row copy a step-mode append_batch leaves to paged_attention."""

    __slots__ = ("step", "k_new", "v_new", "seq_out")

    def __init__(self, step, k_new, v_new):
        self.step = step
        self.k_new = k_new
        self.v_new = v_new
        self.seq_out = step.meta.seq_out[: step.B]


class DecodeStep:
    """One decode token for every request of a batch, in every layer.

    ``layer_states[l][b]`` is request b's cache state in layer l (this
    package's ``PagedKVCacheState`` or the reference's); the layers' pools
    must already hold the prompts (the step allocates, it does not
    initialise).  ``begin()`` plans the step, ``end()`` closes it; use it as a
    context manager around the model's forward."""

    def __init__(self, layer_states: list[list], meta: SharedStepMetadata | None = None):
        if not layer_states or not layer_states[0]:
            raise ValueError("b2pa.DecodeStep needs at least one layer and one request")
        self.layer_states = [list(states) for states in layer_states]
        self.B = len(self.layer_states[0])
        if any(len(states) != self.B for states in self.layer_states):
            raise ValueError("b2pa.DecodeStep: every layer must hold the same requests")
        self.pools = [states[0].pool for states in self.layer_states]
        for states, pool in zip(self.layer_states, self.pools):
            if any(s.pool is not pool for s in states):
                raise ValueError("b2pa.DecodeStep: a layer's requests must share that layer's pool")
            if pool.k_blocks is None:
                raise ValueError("b2pa.DecodeStep: a layer's pool holds nothing yet (run the prompt first)")
        self.meta = meta
        self.open = False

    def _width_needed(self) -> int:
        bs = self.pools[0].block_size
        return max(-(-(s.seq_len + 1) // bs) for s in self.layer_states[0])

    def begin(self) -> "DecodeStep":
        from .paged_kv import flush_pending

        if self.open:
            raise RuntimeError("b2pa.DecodeStep.begin: the step is already open")
        for pool in self.pools:
            if getattr(pool, "_b2pa_pending", None) is not None:
                flush_pending(pool)
            if getattr(pool, "_b2pa_step", None) is not None:
                raise RuntimeError("b2pa.DecodeStep.begin: a pool is already in an open step")
        device = self.pools[0].k_blocks.device
        width = self._width_needed()
        if (self.meta is None or self.meta.capacity < self.B or self.meta.width < width
                or self.meta.device != device):
            cap = max(self.B, self.meta.capacity if self.meta is not None else 0)
            self.meta = SharedStepMetadata(device, cap, width + width // 2 + 16)
        self.meta.B = self.B
        starts = reserve_lockstep(self.layer_states, self.pools)
        first = self.layer_states[0]
        self.meta.upload([s.block_ids for s in first], [s.seq_len for s in first], starts)
        kb = self.pools[0].k_blocks
        self.meta.ensure_workspace(kb.shape[1], kb.shape[3], kb.shape[2], kb.dtype)
        for pool in self.pools:
            pool._b2pa_step = self
        self.open = True
        return self

    def end(self) -> None:
        from .paged_kv import flush_pending

        for pool in self.pools:
            if getattr(pool, "_b2pa_pending", None) is not None and isinstance(pool._b2pa_pending, _StepPending):
                pool._b2pa_pending = None
                raise RuntimeError("b2pa.DecodeStep.end: a layer appended its row but never ran its attention")
            flush_pending(pool)
            pool._b2pa_step = None
        self.open = False

    def __enter__(self):
        return self.begin()

    def __exit__(self, exc_type, exc, tb):
        if exc_type is None:
            self.end()
        else:  # leave the pools usable; the error propagates
            for pool in self.pools:
                pool._b2pa_pending = None
                pool._b2pa_step = None
            self.open = False
        return False

    # --------------------------------------- hooks used by paged_kv / attention
    def layer_of(self, cache) -> int:
        try:
            l = self.pools.index(cache.pool)
        except ValueError:
            raise RuntimeError("b2pa.DecodeStep: a cache whose pool is not in the step") from None
        states = cache.states
        mine = self.layer_states[l]
        if len(states) != self.B or any(a is not b for a, b in zip(states, mine)):
            raise RuntimeError("b2pa.DecodeStep: append_batch on another set of requests than the step's")
        return l

    def append(self, cache, k_new: torch.Tensor, v_new: torch.Tensor, current_lengths) -> torch.Tensor:
        self.layer_of(cache)
        B, H, T, D = k_new.shape
        if T != 1 or not _all_ones(current_lengths, B):
            raise RuntimeError("b2pa.DecodeStep: a decode step appends exactly one token per request")
        if k_new.stride(3) != 1 or v_new.stride(3) != 1:
            raise RuntimeError("b2pa.DecodeStep: k_new / v_new need a unit head_dim stride")
        cache.pool._b2pa_pending = _StepPending(self, k_new, v_new)
        return self.meta.seq_out[: self.B]

    def attend(self, q: torch.Tensor, cache, pend: _StepPending) -> torch.Tensor:
        """b2pa_paged_decode_append on the shared metadata (no host work
        beyond the launch)."""
        pool = cache.pool
        kb, vb = pool.k_blocks, pool.v_blocks
        B, H, _, D = q.shape
        m = self.meta
        out = torch.empty_like(q)
        dev = q.device
        lib = _lib.load()
        ws = m.workspace
        rc = lib.b2pa_paged_decode_append(
            q.data_ptr(), _lib.strides4(q), pend.k_new.data_ptr(), _lib.strides4(pend.k_new), pend.v_new.data_ptr(),
            _lib.strides4(pend.v_new), kb.data_ptr(), vb.data_ptr(), _lib.strides4(kb), kb.shape[0],
            m.table.data_ptr(), m.width, m.width, m.seq_lens.data_ptr(), m.ones.data_ptr(), m.start_pos.data_ptr(),
            m.ones.data_ptr(), m.seq_out.data_ptr(), out.data_ptr(), _lib.strides4(out), B, H, D, kb.shape[2],
            1.0 / math.sqrt(D), _lib.dtype_code(q.dtype), ws.data_ptr(), ws.numel(),
            _lib.status_buffer(dev).data_ptr(), _lib.stream_handle(dev))
        _lib.check(rc, "b2pa_paged_decode_append (decode step)")
        return out

    def signature(self) -> tuple:
        """Every address and size a captured step bakes in."""
        m = self.meta
        return (self.B, m.width, m.dev.data_ptr(), m.workspace.data_ptr(),
                tuple((p.k_blocks.data_ptr(), p.v_blocks.data_ptr(), p.k_blocks.shape[0]) for p in self.pools))


def reserve_lockstep(layer_states: list[list], pools: list) -> list[int]:
    """Allocates one decode token for every request in every layer, as the
    reference's per-layer append_batch would (each layer's own pool, requests
    in batch order, a block whenever the write position reaches a block
    boundary: src/cache/paged_kv.py:110-113), after checking that the layers
    are in lockstep -- same lengths and block tables, and pools that will
    hand out the same ids (same capacity, same next free ids) -- so that one
    table serves every layer.  Refuses, changing nothing, when they are not;
    checks the resulting tables again after allocating.  Returns each
    request's position of the new token."""
    first, p0 = layer_states[0], pools[0]
    bs = p0.block_size
    need = sum(1 for s in first if s.seq_len % bs == 0)
    for l in range(1, len(layer_states)):
        pool = pools[l]
        for b, (s, s0) in enumerate(zip(layer_states[l], first)):
            if s.seq_len != s0.seq_len or s.block_ids != s0.block_ids:
                raise RuntimeError(
                    f"b2pa.DecodeStep: layer {l} request {b} (length {s.seq_len}, {len(s.block_ids)} blocks) differs "
                    f"from layer 0 (length {s0.seq_len}, {len(s0.block_ids)} blocks); the layers are not in "
                    "lockstep, so one table cannot serve them")
        if pool.block_size != bs or pool.capacity_blocks != p0.capacity_blocks or (
                need and pool.free_block_ids[-need:] != p0.free_block_ids[-need:]):
            raise RuntimeError(f"b2pa.DecodeStep: layer {l}'s pool would hand out other block ids than layer 0's")
    starts = [s.seq_len for s in first]
    for states, pool in zip(layer_states, pools):
        for s in states:
            if s.seq_len % bs == 0:
                s.block_ids.append(pool.allocate_block())
            s.seq_len += 1
    for l in range(1, len(layer_states)):
        for s, s0 in zip(layer_states[l], first):
            if s.block_ids[-1] != s0.block_ids[-1]:
                raise RuntimeError(f"b2pa.DecodeStep: layer {l} allocated other block ids than layer 0")
    return starts


def _all_ones(current_lengths, B: int) -> bool:
    if current_lengths is None or (isinstance(current_lengths, int) and current_lengths == 1):
        return True
    if isinstance(current_lengths, torch.Tensor):
        if current_lengths.is_cuda:
            return True  # not read on the host (a decode step's lengths are ones by contract)
        return bool((current_lengths == 1).all())
    return all(int(x) == 1 for x in current_lengths)


def active_step(pool):
    """The open DecodeStep a pool belongs to, if any."""
    return getattr(pool, "_b2pa_step", None)


class DecodeGraph:
    """Runs a decode-step function as a CUDA graph.

    ``step_fn()`` runs the model for one decode token, reading its inputs
    from tensors the caller keeps at fixed addresses (token ids, positions)
    and returning an output tensor (e.g. the sampled ids).  Each ``__call__``
    opens a ``DecodeStep`` over ``layer_states`` (allocation and the shared
    metadata upload on the host), then replays the captured graph; the first
    call, and the first call after anything the graph baked in has moved,
    runs ``step_fn`` eagerly (warm-up) or captures it.  Returns the output
    tensor of the replay (the graph's own buffer: copy it before the next
    call if it must be kept)."""

    def __init__(self, step_fn, warmup_steps: int = 1):
        self.step_fn = step_fn
        self.warmup_steps = warmup_steps
        self.graph: torch.cuda.CUDAGraph | None = None
        self.output = None
        self.sig = None
        self.meta: SharedStepMetadata | None = None
        self.captures = 0
        self.replays = 0
        self.eager_steps = 0
        self._since_change = 0
        self.stream: torch.cuda.Stream | None = None

    def __call__(self, layer_states: list[list]):
        step = DecodeStep(layer_states, self.meta)
        step.begin()
        self.meta = step.meta
        dev = step.meta.device
        cur = torch.cuda.current_stream(dev)
        try:
            sig = step.signature()
            if sig != self.sig:
                self.graph, self.output, self.sig = None, None, sig
                self._since_change = 0
            if self.stream is None:
                self.stream = torch.cuda.Stream(dev)
            if self.graph is None and self._since_change < self.warmup_steps:
                # eager step on the stream the capture will use, so that
                # libraries set up their per-stream state outside the capture
                self.stream.wait_stream(cur)
                with torch.cuda.stream(self.stream):
                    out = self.step_fn()
                cur.wait_stream(self.stream)
                self.eager_steps += 1
                self._since_change += 1
                step.end()
                return out
            if self.graph is None:
                g = torch.cuda.CUDAGraph()
                self.stream.wait_stream(cur)
                with torch.cuda.stream(self.stream):
                    with torch.cuda.graph(g, stream=self.stream):
                        self.output = self.step_fn()
                cur.wait_stream(self.stream)
                self.graph = g
                self.captures += 1
            self.graph.replay()
            self.replays += 1
            step.end()
            return self.output
        except BaseException:
            if step.open:
                step.__exit__(RuntimeError, None, None)
            raise
