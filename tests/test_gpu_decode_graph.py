"""The decode step as a CUDA graph (b2pa.DecodeGraph) on the GPU: one block
table shared by all layers per step (allocation checked to be in lockstep),
the model's whole decode step -- embeddings, projections, attention with its
fused KV append, MLP, lm_head, argmax -- captured once and replayed.

* config[0] (batch 1, 128-token prompt, 128 greedy tokens): tokens identical
  to the eager run and to the reference's own CPU run (golden); logits at
  every step within rtol 1e-4 / atol 1e-5 of the eager run; every layer's
  pool bit-identical to the eager run's; tokens/s with and without the graph;
* a batch of three prompts of different lengths (padded prefill) decoded
  with and without the graph: tokens and pools identical;
* pools that grow during decoding (torch.cat moves them): the graph is
  captured again and the tokens stay identical."""
from __future__ import annotations

import json
import time

import numpy as np
import pytest
import torch

from oracle import model as om
from tests._helpers import load_golden

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int32).numpy()


def _prefill(model, prompt, lengths):
    """The prompt chunk, as generate_with_cache runs it; returns the first
    sampled ids and the per-layer cache states [layer][request]."""
    B = prompt.shape[0]
    cur = torch.tensor(lengths, dtype=torch.long, device=prompt.device)
    logits, caches = model(prompt, position_offset=0, current_lengths=cur)
    nxt = torch.argmax(logits[torch.arange(B, device=prompt.device), cur - 1, :], dim=-1)
    layer_states = [list(c.states) if hasattr(c, "states") else [c] for c in caches]
    return nxt, layer_states


def _decode_eager(model, nxt, layer_states, lengths, steps):
    """Plain per-step model calls (the b2pa backend's ordinary path)."""
    B = len(lengths)
    dev = nxt.device
    toks, logits_all = [], []
    for step in range(steps):
        pos = torch.tensor([L + step for L in lengths], dtype=torch.long, device=dev)
        caches = [model.backend.batch_cls(states=list(st), pool=st[0].pool) for st in layer_states]
        logits, _ = model(nxt.view(B, 1), kv_caches=caches, position_offset=pos, current_lengths=1)
        logits_all.append(logits[:, -1, :].float().cpu())
        nxt = torch.argmax(logits[:, -1, :], dim=-1)
        toks.append(nxt.cpu())
    torch.cuda.synchronize()
    return torch.stack(toks, 1), logits_all


def _decode_graph(model, nxt, layer_states, lengths, steps):
    import b2pa

    B = len(lengths)
    dev = nxt.device
    ids = torch.zeros(B, 1, dtype=torch.long, device=dev)
    pos = torch.zeros(B, dtype=torch.long, device=dev)
    base = torch.tensor(lengths, dtype=torch.long, device=dev)
    caches = [model.backend.batch_cls(states=list(st), pool=st[0].pool) for st in layer_states]

    def step_fn():
        logits, _ = model(ids, kv_caches=caches, position_offset=pos, current_lengths=1)
        last = logits[:, -1, :]
        return last, torch.argmax(last, dim=-1)

    graph = b2pa.DecodeGraph(step_fn)
    ids.copy_(nxt.view(B, 1))
    toks, logits_all = [], []
    for step in range(steps):
        torch.add(base, step, out=pos)
        last, nxt_t = graph(layer_states)
        logits_all.append(last.float().cpu())
        toks.append(nxt_t.cpu())
        ids.copy_(nxt_t.view(B, 1))
    torch.cuda.synchronize()
    return torch.stack(toks, 1), logits_all, graph


def _timed_tokens(run):
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = run()
    torch.cuda.synchronize()
    return out, time.perf_counter() - t0


@torch.no_grad()
def test_config0_decode_graph(cuda_device):
    import b2pa

    g = load_golden("model_config0")
    prev = b2pa.set_fused_append(True)
    try:
        runs = {}
        for mode in ("eager", "graph", "eager", "graph"):  # second pair timed warm
            model, prompt = om.config0_model(om.b2pa_backend(), cuda_device)
            nxt, layer_states = _prefill(model, prompt, [128])
            first = nxt.cpu()
            if mode == "eager":
                (toks, logits), secs = _timed_tokens(lambda: _decode_eager(model, nxt, layer_states, [128], 127))
                graph = None
            else:
                (toks, logits, graph), secs = _timed_tokens(
                    lambda: _decode_graph(model, nxt, layer_states, [128], 127))
            runs[mode] = (torch.cat([first.view(1, 1), toks], 1), logits, model, secs, graph)
    finally:
        b2pa.set_fused_append(prev)
    te, le, me, se, _ = runs["eager"]
    tg, lg, mg, sg, graph = runs["graph"]
    assert np.array_equal(te.numpy(), g["tokens"]) and np.array_equal(tg.numpy(), g["tokens"])
    for a, b in zip(le, lg):
        np.testing.assert_allclose(b.numpy(), a.numpy(), rtol=1e-4, atol=1e-5)
    for pe, pg in zip(me.pools, mg.pools):
        assert np.array_equal(_bits(pe.k_blocks), _bits(pg.k_blocks))
        assert np.array_equal(_bits(pe.v_blocks), _bits(pg.v_blocks))
        assert pe.free_block_ids == pg.free_block_ids
    assert graph.captures == 1 and graph.replays == 126 and graph.eager_steps == 1
    assert b2pa.read_status(cuda_device) == 0
    print(json.dumps({"config": "BASELINE config[0] decode: 127 greedy steps after the 128-token prompt, batch 1, FP32",
                      "eager_decode_s": se, "graph_decode_s": sg,
                      "eager_tokens_per_s": 127 / se, "graph_tokens_per_s": 127 / sg,
                      "graph_ms_per_token": sg / 127 * 1e3}))


@torch.no_grad()
@pytest.mark.parametrize("initial_blocks", [64, 2], ids=["no_growth", "growth_recaptures"])
def test_batched_ragged_decode_graph(cuda_device, initial_blocks):
    import b2pa

    lengths = [40, 25, 33]
    prev = b2pa.set_fused_append(True)
    try:
        outs = []
        for use_graph in (False, True):
            om.set_seed(7)
            model = om.TinyLM(500, 128, 4, 3, 256, 256, om.b2pa_backend(), kv_block_size=16,
                              kv_pool_initial_blocks=initial_blocks, kv_pool_growth_factor=2.0).to(cuda_device).eval()
            prompt = torch.randint(0, 500, (3, 40), generator=torch.Generator().manual_seed(3)).to(cuda_device)
            nxt, layer_states = _prefill(model, prompt, lengths)
            if use_graph:
                toks, logits, graph = _decode_graph(model, nxt, layer_states, lengths, 60)
            else:
                toks, logits = _decode_eager(model, nxt, layer_states, lengths, 60)
                graph = None
            outs.append((toks, logits, model, graph))
    finally:
        b2pa.set_fused_append(prev)
    (te, le, me, _), (tg, lg, mg, graph) = outs
    assert torch.equal(te, tg)
    for a, b in zip(le, lg):
        np.testing.assert_allclose(b.numpy(), a.numpy(), rtol=1e-4, atol=1e-5)
    for pe, pg in zip(me.pools, mg.pools):
        assert pe.capacity_blocks == pg.capacity_blocks
        assert np.array_equal(_bits(pe.k_blocks), _bits(pg.k_blocks))
        assert np.array_equal(_bits(pe.v_blocks), _bits(pg.v_blocks))
    if initial_blocks == 2:
        assert graph.captures >= 2  # the pools moved when they grew
    else:
        assert graph.captures == 1
    assert b2pa.read_status(cuda_device) == 0
