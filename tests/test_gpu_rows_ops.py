"""The decode step's non-attention operations on the GPU (b2pa_rows_linear,
b2pa_rows_embed, b2pa_rows_argmax, through the C ABI) against torch in
float64 on the same fp32 inputs, and b2pa.FusedDecoder -- the whole decode
step of the config[0] model on b2pa kernels, eager and as a CUDA graph --
against the model's own path: greedy tokens identical to the reference's
(golden), logits within rtol 1e-4 / atol 1e-5 at every step."""
from __future__ import annotations

import json
import time

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import model as om
from tests._helpers import load_golden

pytestmark = pytest.mark.gpu


def _lib():
    from b2pa import _lib

    return _lib, _lib.load()


@pytest.mark.parametrize("M", [1, 3, 8, 16])
@pytest.mark.parametrize("K,N", [(512, 1536), (512, 2048), (2048, 512), (512, 5000), (64, 36)])
@pytest.mark.parametrize("mode", ["plain", "ln_gelu", "residual"])
def test_rows_linear_matches_float64(cuda_device, M, K, N, mode):
    L, lib = _lib()
    g = torch.Generator(device=cuda_device).manual_seed(M * 1000 + K + N)
    xs = K + 8  # a padded row stride
    xbuf = torch.randn(M, xs, generator=g, device=cuda_device)
    x = xbuf[:, :K]
    w = torch.randn(N, K, generator=g, device=cuda_device) / K ** 0.5
    b = torch.randn(N, generator=g, device=cuda_device)
    gam = torch.randn(K, generator=g, device=cuda_device)
    bet = torch.randn(K, generator=g, device=cuda_device)
    y0 = torch.randn(M, N, generator=g, device=cuda_device)
    y = y0.clone()
    ln = mode == "ln_gelu"
    rc = lib.b2pa_rows_linear(x.data_ptr(), xs, M, K, gam.data_ptr() if ln else None, bet.data_ptr() if ln else None,
                              1e-5, w.data_ptr(), b.data_ptr(), N, 1 if ln else 0, y.data_ptr(), N,
                              1 if mode == "residual" else 0, L.status_buffer(cuda_device).data_ptr(),
                              L.stream_handle(cuda_device))
    L.check(rc, "rows_linear")
    x64 = x.double()
    if ln:
        x64 = F.layer_norm(x64, (K,), gam.double(), bet.double(), 1e-5)
    r = x64 @ w.double().T + b.double()
    if ln:
        r = F.gelu(r)
    ref = y0.double() + r if mode == "residual" else r
    np.testing.assert_allclose(y.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5, atol=1e-5)


def test_rows_linear_refuses_bad_shapes(cuda_device):
    L, lib = _lib()
    x = torch.zeros(17, 64, device=cuda_device)
    args = lambda M, K, stride: lib.b2pa_rows_linear(x.data_ptr(), stride, M, K, None, None, 0.0, x.data_ptr(), None,
                                                     4, 0, x.data_ptr(), 64, 0, None, None)
    assert args(17, 64, 64) == -1      # more than 16 rows
    assert args(2, 62, 64) == -2       # K not a multiple of 4
    assert args(2, 64, 62) == -2       # row stride below K / not 16-byte rows
    assert args(0, 64, 64) == 0


def test_rows_embed_and_argmax(cuda_device):
    L, lib = _lib()
    st = L.status_buffer(cuda_device)
    tok = torch.randn(100, 64, device=cuda_device)
    pos = torch.randn(50, 64, device=cuda_device)
    ids = torch.tensor([3, 99, 0, 7], device=cuda_device)
    p = torch.tensor([0, 49, 5, 5], device=cuda_device)
    x = torch.empty(4, 64, device=cuda_device)
    L.check(lib.b2pa_rows_embed(ids.data_ptr(), p.data_ptr(), 4, tok.data_ptr(), 100, pos.data_ptr(), 50, 64,
                                x.data_ptr(), 64, st.data_ptr(), L.stream_handle(cuda_device)), "embed")
    assert torch.equal(x, tok[ids] + pos[p])
    assert L.read_status(cuda_device) == 0
    bad = torch.tensor([3, 100, 0, 7], device=cuda_device)  # out of the table: zero row, status set
    L.check(lib.b2pa_rows_embed(bad.data_ptr(), p.data_ptr(), 4, tok.data_ptr(), 100, pos.data_ptr(), 50, 64,
                                x.data_ptr(), 64, st.data_ptr(), L.stream_handle(cuda_device)), "embed")
    assert torch.equal(x[1], torch.zeros(64, device=cuda_device)) and torch.equal(x[0], tok[3] + pos[0])
    assert L.read_status(cuda_device) == L.STATUS_CODES["B2PA_ERR_INVALID_ARGUMENT"]
    L.clear_status(cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(1)
    logits = torch.randn(6, 5003, generator=g, device=cuda_device)
    logits[1, 17] = logits[1, 4000] = 100.0                     # a tie: the first index
    logits[2] = -float("inf")                                  # all -inf: index 0
    logits[3, 5002] = 50.0                                     # the last column
    logits[4, :] = 7.0                                         # all equal: index 0
    out = torch.empty(6, dtype=torch.int64, device=cuda_device)
    L.check(lib.b2pa_rows_argmax(logits.data_ptr(), 5003, 6, 5003, out.data_ptr(), None,
                                 L.stream_handle(cuda_device)), "argmax")
    assert out.tolist() == torch.argmax(logits, dim=-1).tolist()
    assert out.tolist()[1:5] == [17, 0, 5002, 0]


def _prefill(model, prompt):
    logits, caches = model(prompt, position_offset=0,
                           current_lengths=torch.full((prompt.shape[0],), prompt.shape[1], device=prompt.device))
    return torch.argmax(logits[:, -1, :], dim=-1), caches


@torch.no_grad()
def test_fused_decoder_config0(cuda_device):
    import b2pa

    gold = load_golden("model_config0")
    prev = b2pa.set_fused_append(True)
    try:
        # the model's own path (torch modules + b2pa attention), per-step logits
        model, prompt = om.config0_model(om.b2pa_backend(), cuda_device)
        toks_m, logits_m, _ = om.generate_with_cache(model, prompt, 128, keep_logits=True)
        results = {}
        for mode in ("eager", "graph"):
            model, prompt = om.config0_model(om.b2pa_backend(), cuda_device)
            dec = b2pa.FusedDecoder(model, max_batch=1)
            nxt, caches = _prefill(model, prompt)
            layer_states = [[c] for c in caches]
            batches = [model.backend.batch_cls(states=[c], pool=c.pool) for c in caches]
            ids = nxt.clone()
            pos = torch.zeros(1, dtype=torch.int64, device=cuda_device)
            toks, logits = [nxt.cpu()], [None]
            step_fn = lambda: dec.step(ids, pos, batches)
            graph = b2pa.DecodeGraph(step_fn) if mode == "graph" else None
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for s in range(1, 128):
                pos.fill_(128 + s - 1)
                if graph is None:
                    with b2pa.DecodeStep(layer_states):
                        lg, nx = step_fn()
                else:
                    lg, nx = graph(layer_states)
                logits.append(lg.float().cpu())
                toks.append(nx.cpu())
                ids.copy_(nx)
            torch.cuda.synchronize()
            results[mode] = (torch.stack(toks, 1), logits, time.perf_counter() - t0, graph)
    finally:
        b2pa.set_fused_append(prev)
    for mode, (toks, logits, secs, graph) in results.items():
        assert np.array_equal(toks.numpy(), gold["tokens"]), mode
        for s in range(1, 128):
            np.testing.assert_allclose(logits[s].numpy(), logits_m[s].numpy(), rtol=1e-4, atol=1e-5)
    assert results["graph"][3].captures == 1
    assert b2pa.read_status(cuda_device) == 0


@torch.no_grad()
def test_fused_decoder_batched_ragged(cuda_device):
    """Three requests of different lengths in one step (padded prefill), 40
    greedy steps on FusedDecoder under a CUDA graph against the model's own
    decode path: tokens identical, logits within the fp32 tolerance."""
    import b2pa

    lengths = [40, 25, 33]
    prev = b2pa.set_fused_append(True)
    outs = []
    try:
        for use_fused in (False, True):
            om.set_seed(7)
            model = om.TinyLM(500, 128, 4, 3, 256, 256, om.b2pa_backend(), kv_block_size=16).to(cuda_device).eval()
            prompt = torch.randint(0, 500, (3, 40), generator=torch.Generator().manual_seed(3)).to(cuda_device)
            cur = torch.tensor(lengths, device=cuda_device)
            lg, caches = model(prompt, position_offset=0, current_lengths=cur)
            nxt = torch.argmax(lg[torch.arange(3, device=cuda_device), cur - 1, :], dim=-1)
            layer_states = [list(c.states) for c in caches]
            batches = [model.backend.batch_cls(states=list(st), pool=st[0].pool) for st in layer_states]
            toks, logits = [], []
            if use_fused:
                dec = b2pa.FusedDecoder(model, max_batch=4)
                ids, pos = nxt.clone(), torch.zeros(3, dtype=torch.int64, device=cuda_device)
                graph = b2pa.DecodeGraph(lambda: dec.step(ids, pos, batches))
            for s in range(40):
                p = torch.tensor([L + s for L in lengths], device=cuda_device)
                if use_fused:
                    pos.copy_(p)
                    lgs, nx = graph(layer_states)
                    ids.copy_(nx)
                else:
                    bt = [model.backend.batch_cls(states=list(st), pool=st[0].pool) for st in layer_states]
                    out, _ = model(nxt.view(3, 1), kv_caches=bt, position_offset=p, current_lengths=1)
                    lgs = out[:, -1, :]
                    nx = torch.argmax(lgs, dim=-1)
                    nxt = nx
                logits.append(lgs.float().cpu())
                toks.append(nx.cpu())
            outs.append((torch.stack(toks, 1), logits))
    finally:
        b2pa.set_fused_append(prev)
    assert torch.equal(outs[0][0], outs[1][0])
    for a, b in zip(outs[0][1], outs[1][1]):
        np.testing.assert_allclose(b.numpy(), a.numpy(), rtol=1e-4, atol=1e-5)
    assert b2pa.read_status(cuda_device) == 0


@torch.no_grad()
def test_decode_step_throughput_config0(cuda_device):
    """config[0] decode (127 greedy steps after the prompt, batch 1) four
    ways, with the tokens kept on the device and one synchronisation at the
    end, steps 3-127 timed: the model's own step (torch modules + b2pa attention), the same as a
    CUDA graph, FusedDecoder, and FusedDecoder as a CUDA graph.  Tokens must
    equal the reference's (golden) every way; prints tokens/s."""
    import b2pa

    gold = load_golden("model_config0")["tokens"]
    prev = b2pa.set_fused_append(True)
    report = {"config": "BASELINE config[0] decode: 127 greedy steps after the 128-token prompt, batch 1, FP32; "
                        "tokens kept on the device, steps 3-127 timed (after a graph's warm-up step and "
                        "capture), one host synchronisation at the end"}
    try:
        for name in ("model_eager", "model_graph", "fused_eager", "fused_graph", "model_eager", "model_graph",
                     "fused_eager", "fused_graph"):
            model, prompt = om.config0_model(om.b2pa_backend(), cuda_device)
            nxt, caches = _prefill(model, prompt)
            layer_states = [[c] for c in caches]
            batches = [model.backend.batch_cls(states=[c], pool=c.pool) for c in caches]
            ids = nxt.clone()
            pos = torch.zeros(1, dtype=torch.int64, device=cuda_device)
            toks = torch.empty(1, 128, dtype=torch.int64, device=cuda_device)
            toks[:, 0] = nxt
            if name.startswith("fused"):
                dec = b2pa.FusedDecoder(model, max_batch=1)
                step_fn = lambda: dec.step(ids, pos, batches)[1]
            else:
                def step_fn():
                    logits, _ = model(ids.view(1, 1), kv_caches=batches, position_offset=pos, current_lengths=1)
                    return torch.argmax(logits[:, -1, :], dim=-1)
            graph = b2pa.DecodeGraph(step_fn) if name.endswith("graph") else None
            t0 = None
            for s in range(1, 128):
                if s == 3:  # steps 1-2 (a graph's warm-up and capture) are not timed
                    torch.cuda.synchronize()
                    t0 = time.perf_counter()
                pos.fill_(128 + s - 1)
                if graph is not None:
                    nx = graph(layer_states)
                elif name.startswith("fused"):
                    with b2pa.DecodeStep(layer_states):
                        nx = step_fn()
                else:
                    nx = step_fn()
                toks[:, s] = nx
                ids.copy_(nx)
            torch.cuda.synchronize()
            secs = time.perf_counter() - t0
            assert np.array_equal(toks.cpu().numpy(), gold), name
            report[name + "_tokens_per_s"] = 125 / secs  # the second (warm) run of each way is kept
            if graph is not None:
                # device time of one step: the captured step replayed back to back (it rewrites the
                # last step's rows with the same values and recomputes the same outputs)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(50):
                    graph.graph.replay()
                b.record()
                torch.cuda.synchronize()
                report[name + "_device_us_per_step"] = a.elapsed_time(b) / 50 * 1e3
    finally:
        b2pa.set_fused_append(prev)
    assert b2pa.read_status(cuda_device) == 0
    print(json.dumps(report))
