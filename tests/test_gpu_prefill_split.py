"""Chunked prefill at the edges of its work split, on the GPU through the C ABI.

The tensor-core kernel runs one CTA per (128 query rows, head, sequence) and
splits the key range of those CTAs across several when they alone would
leave SMs idle, merging the pieces in a combine launch.  These cases stress
that: one 128-row query tile over a 19,872-token prefix (the key range cut
into many pieces), many small units (64 sequences x 8 heads of short
chunks, some empty), ragged query tiles, and repeated calls and CUDA-graph
replays on one workspace that starts as random bytes.  Checked against the
CPU oracle (fp32: rtol 1e-4 / atol 1e-5; 16-bit: 2e-2) and, across repeats,
value for value.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from b2pa import _lib
from oracle import oracle as orc
from tests._helpers import TOL, random_tables, strided_q

pytestmark = pytest.mark.gpu


def _i32(v, device):
    return torch.tensor(list(v), dtype=torch.int32, device=device)


def _problem(device, *, B, H, D, bs, T, dtype, prefixes, curs, seed):
    rng = np.random.default_rng(seed)
    gen = torch.Generator().manual_seed(seed)
    lens = [p + c for p, c in zip(prefixes, curs)]
    NB = sum(-(-L // bs) for L in lens) + 3
    kp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    vp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    tables = random_tables(rng, lens, NB, bs)
    width = max(max(len(t) for t in tables), 1)
    table = np.full((B, width), -1, dtype=np.int32)
    for b, t in enumerate(tables):
        table[b, :len(t)] = t
    q = strided_q(B, H, T, D, dtype, device, gen)
    return dict(B=B, H=H, D=D, bs=bs, T=T, dtype=dtype, kp=kp, vp=vp, tables=tables, lens=lens, curs=list(curs),
                table=torch.from_numpy(table).to(device), width=width, q=q, NB=NB,
                seq=_i32(lens, device), cur=_i32(curs, device))


def _workspace(pr, device, seed=0):
    n = _lib.load().b2pa_paged_prefill_workspace_size(pr["B"], pr["H"], pr["T"], pr["D"], pr["width"], pr["bs"],
                                                      _lib.dtype_code(pr["dtype"]))
    # random bytes: nothing in the workspace may be assumed initialised (a
    # call that needs none still gets a buffer)
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randint(0, 256, (max(n, 256),), dtype=torch.uint8, device=device, generator=g)


def _call(pr, out, ws, device):
    lib = _lib.load()
    return lib.b2pa_paged_prefill(
        pr["q"].data_ptr(), _lib.strides4(pr["q"]), pr["kp"].data_ptr(), pr["vp"].data_ptr(), _lib.strides4(pr["kp"]),
        pr["NB"], pr["table"].data_ptr(), pr["width"], pr["width"], pr["seq"].data_ptr(), pr["cur"].data_ptr(),
        out.data_ptr(), _lib.strides4(out), pr["B"], pr["H"], pr["T"], pr["D"], pr["bs"], 1.0 / math.sqrt(pr["D"]),
        _lib.dtype_code(pr["dtype"]), ws.data_ptr(), ws.numel(), _lib.status_buffer(device).data_ptr(),
        _lib.stream_handle(device))


def _oracle(pr):
    return orc.paged_attention_c(pr["q"].float().cpu().numpy(), pr["kp"].float().cpu().numpy(),
                                 pr["vp"].float().cpu().numpy(), pr["tables"], pr["lens"], pr["curs"])


def _run_checked(pr, device, repeats=3):
    _lib.clear_status(device)
    ws = _workspace(pr, device)
    outs = []
    for _ in range(repeats):
        out = torch.full_like(pr["q"], float("nan"))
        _lib.check(_call(pr, out, ws, device), "b2pa_paged_prefill")
        outs.append(out)
    torch.cuda.synchronize()
    assert _lib.read_status(device) == 0
    np.testing.assert_allclose(outs[0].float().cpu().numpy(), _oracle(pr), **TOL[pr["dtype"]])
    for o in outs[1:]:  # same plan, same merge order: the same values
        assert torch.equal(o, outs[0])
    return outs[0], ws


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_one_query_tile_long_prefix(cuda_device, dtype):
    # 128 query rows over a 19,872-token prefix: 313 key tiles, one query
    # tile -- the key range is cut into many pieces and merged
    pr = _problem(cuda_device, B=1, H=1, D=64, bs=16, T=128, dtype=dtype, prefixes=[19872], curs=[128], seed=31)
    _run_checked(pr, cuda_device)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("bs", [8, 32])
def test_many_small_units_per_cta(cuda_device, dtype, bs):
    # 64 sequences x 8 heads of short chunks over short prefixes: 512 CTAs
    # of 1-3 key tiles, some sequences empty
    rng = np.random.default_rng(7 + bs)
    curs = rng.integers(0, 21, size=64)
    prefixes = rng.integers(0, 150, size=64) * (curs > 0)
    pr = _problem(cuda_device, B=64, H=8, D=64, bs=bs, T=20, dtype=dtype, prefixes=prefixes.tolist(),
                  curs=curs.tolist(), seed=bs)
    _run_checked(pr, cuda_device)


@pytest.mark.parametrize("D", [64, 128])
def test_ragged_query_tiles(cuda_device, D):
    # three query tiles per sequence (the last one partly past T), unequal
    # prefixes: CTAs of very different key ranges
    pr = _problem(cuda_device, B=5, H=3, D=D, bs=16, T=300, dtype=torch.bfloat16,
                  prefixes=[0, 2500, 40, 900, 0], curs=[300, 300, 170, 1, 0], seed=D)
    _run_checked(pr, cuda_device)


def test_graph_replays_are_repeatable(cuda_device):
    """Replays of one captured call (with a key-range split and its combine)
    give the eager call's result every time."""
    pr = _problem(cuda_device, B=3, H=8, D=64, bs=16, T=256, dtype=torch.bfloat16, prefixes=[700, 60, 3000],
                  curs=[256, 256, 100], seed=11)
    ref, ws = _run_checked(pr, cuda_device, repeats=1)
    out = torch.zeros_like(pr["q"])
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            rc = _lib.load().b2pa_paged_prefill(
                pr["q"].data_ptr(), _lib.strides4(pr["q"]), pr["kp"].data_ptr(), pr["vp"].data_ptr(),
                _lib.strides4(pr["kp"]), pr["NB"], pr["table"].data_ptr(), pr["width"], pr["width"],
                pr["seq"].data_ptr(), pr["cur"].data_ptr(), out.data_ptr(), _lib.strides4(out), pr["B"], pr["H"],
                pr["T"], pr["D"], pr["bs"], 1.0 / math.sqrt(pr["D"]), _lib.dtype_code(pr["dtype"]), ws.data_ptr(),
                ws.numel(), _lib.status_buffer(cuda_device).data_ptr(), s.cuda_stream)
    torch.cuda.current_stream().wait_stream(s)
    _lib.check(rc, "b2pa_paged_prefill (capture)")
    for _ in range(4):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert _lib.read_status(cuda_device) == 0
    del g
