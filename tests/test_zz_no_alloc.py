"""b2pa_paged_decode_noalloc: decode for callers that cannot allocate device
memory (the scratch lives in a fixed array inside libb2pa.so).

Checks, through the C ABI, that two calls in a row give the same results as
b2pa_paged_decode with a caller-provided workspace (within the fp32 / bf16
tolerances of the other decode tests), that the second call is not disturbed
by what the first left in the shared array, and that a problem too large for
the array is refused before any launch.  Kept in its own file, named to be
collected last.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

import b2pa
from b2pa import _lib
from tests._helpers import TOL, random_tables, strided_q

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 << 20  # B2PA_NOALLOC_SCRATCH_BYTES


def _problem(dev, *, B, H, D, bs, dtype, lmin, lmax, seed):
    rng = np.random.default_rng(seed)
    gen = torch.Generator().manual_seed(seed)
    lens = rng.integers(lmin, lmax + 1, size=B).tolist()
    NB = sum(-(-L // bs) for L in lens) + 3
    tables = random_tables(rng, lens, NB, bs)
    max_pages = max(len(t) for t in tables)
    pt = np.full((B, max_pages), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        pt[i, :len(t)] = t
    return dict(
        q=strided_q(B, H, 1, D, dtype, dev, gen),
        k=torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(dev),
        v=torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(dev),
        pt=torch.from_numpy(pt).to(dev), max_pages=max_pages,
        seq=torch.tensor(lens, dtype=torch.int32, device=dev),
        cur=torch.ones(B, dtype=torch.int32, device=dev),
        B=B, H=H, D=D, bs=bs, dtype=dtype,
    )


def _args(p, out):
    return (p["q"].data_ptr(), _lib.strides4(p["q"]), p["k"].data_ptr(), p["v"].data_ptr(), _lib.strides4(p["k"]),
            p["k"].shape[0], p["pt"].data_ptr(), p["pt"].stride(0), p["max_pages"], p["seq"].data_ptr(),
            p["cur"].data_ptr(), out.data_ptr(), _lib.strides4(out), p["B"], p["H"], p["D"], p["bs"],
            1.0 / math.sqrt(p["D"]), _lib.dtype_code(p["dtype"]))


def _with_workspace(lib, p, dev):
    out = torch.empty_like(p["q"])
    n = lib.b2pa_paged_decode_workspace_size(p["B"], p["H"], p["D"], p["max_pages"], p["bs"], _lib.dtype_code(p["dtype"]))
    ws = torch.empty(n, dtype=torch.uint8, device=dev)
    rc = lib.b2pa_paged_decode(*_args(p, out), ws.data_ptr(), n, _lib.status_buffer(dev).data_ptr(),
                               _lib.stream_handle(dev))
    _lib.check(rc, "b2pa_paged_decode")
    return out


def _without_workspace(lib, p, dev):
    out = torch.empty_like(p["q"])
    rc = lib.b2pa_paged_decode_noalloc(*_args(p, out), _lib.status_buffer(dev).data_ptr(), _lib.stream_handle(dev))
    _lib.check(rc, "b2pa_paged_decode_noalloc")
    return out


def test_noalloc_decode_matches_workspace_decode_twice(cuda_device):
    lib = _lib.load()
    b2pa.clear_status(cuda_device)
    # first call: long contexts split into many partials; second call: a
    # different, shorter problem that reuses (and must overwrite) the array
    first = _problem(cuda_device, B=6, H=8, D=128, bs=16, dtype=torch.bfloat16, lmin=3000, lmax=9000, seed=21)
    second = _problem(cuda_device, B=64, H=8, D=64, bs=16, dtype=torch.float32, lmin=128, lmax=1024, seed=22)
    for p in (first, second):
        assert lib.b2pa_paged_decode_workspace_size(p["B"], p["H"], p["D"], p["max_pages"], p["bs"],
                                                    _lib.dtype_code(p["dtype"])) <= SCRATCH_BYTES
    got1 = _without_workspace(lib, first, cuda_device)
    got2 = _without_workspace(lib, second, cuda_device)
    ref1 = _with_workspace(lib, first, cuda_device)
    ref2 = _with_workspace(lib, second, cuda_device)
    torch.cuda.synchronize()
    np.testing.assert_allclose(got1.float().cpu().numpy(), ref1.float().cpu().numpy(), **TOL[torch.bfloat16])
    np.testing.assert_allclose(got2.cpu().numpy(), ref2.cpu().numpy(), **TOL[torch.float32])
    # and once more in the other order, so each call follows a different one
    again1 = _without_workspace(lib, first, cuda_device)
    torch.cuda.synchronize()
    np.testing.assert_allclose(again1.float().cpu().numpy(), ref1.float().cpu().numpy(), **TOL[torch.bfloat16])
    assert b2pa.read_status(cuda_device) == 0


def test_noalloc_rejects_problems_larger_than_the_array(cuda_device):
    lib = _lib.load()
    # 32 sequences x 32 heads x 131072 tokens (item split: 256 streams x 128
    # splits) needs far more than 32 MiB of partials
    B, H, D, bs, max_pages = 32, 32, 128, 16, 8192
    assert lib.b2pa_paged_decode_workspace_size(B, H, D, max_pages, bs, _lib.DTYPE_BF16) > SCRATCH_BYTES
    q = torch.zeros(B, H, 1, D, dtype=torch.bfloat16, device=cuda_device)
    pool = torch.zeros(4, H, bs, D, dtype=torch.bfloat16, device=cuda_device)
    pt = torch.zeros(B, max_pages, dtype=torch.int32, device=cuda_device)
    lens = torch.ones(B, dtype=torch.int32, device=cuda_device)
    out = torch.full_like(q, 7.0)
    rc = lib.b2pa_paged_decode_noalloc(q.data_ptr(), _lib.strides4(q), pool.data_ptr(), pool.data_ptr(),
                                       _lib.strides4(pool), 4, pt.data_ptr(), max_pages, max_pages, lens.data_ptr(),
                                       lens.data_ptr(), out.data_ptr(), _lib.strides4(out), B, H, D, bs,
                                       1.0 / math.sqrt(D), _lib.DTYPE_BF16, None, _lib.stream_handle(cuda_device))
    assert rc == -4
    assert "scratch" in _lib.last_error()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched
