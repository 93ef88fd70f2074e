"""Failure detection on the GPU without faulting it.

The kernels' spin-waits are bounded (1 s of %globaltimer); when one gives up
it records B2PA_ERR_DEVICE_TIMEOUT in the status word and the kernel returns.
b2pa_selftest_wait_timeout reaches that path on purpose (a wait on an
mbarrier nothing arrives at): the status must say so, the kernel must end
after about the limit, and the context must stay usable -- a decode launched
afterwards still matches the oracle.  Bad block ids, the other device-side
failure, are covered by the decode / prefill / append tests."""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import b2pa
from b2pa import _lib
from oracle import oracle as orc
from tests._helpers import TOL, build_cache, random_tables, strided_q

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_the_context_survives(cuda_device):
    lib = _lib.load()
    b2pa.clear_status(cuda_device)
    done = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = lib.b2pa_selftest_wait_timeout(_lib.status_buffer(cuda_device).data_ptr(), done.data_ptr(),
                                        _lib.stream_handle(cuda_device))
    assert rc == 0
    torch.cuda.synchronize()
    secs = time.perf_counter() - t0
    assert done.item() == 2                      # the wait gave up and the kernel went on
    assert b2pa.read_status(cuda_device) == _lib.STATUS_CODES["B2PA_ERR_DEVICE_TIMEOUT"]
    assert 0.9 < secs < 10.0
    with pytest.raises(RuntimeError, match="DEVICE_TIMEOUT"):
        b2pa.raise_on_device_status(cuda_device, "self-test")  # reads and clears
    assert b2pa.read_status(cuda_device) == 0

    # the context is intact: a decode afterwards is correct
    rng = np.random.default_rng(1)
    gen = torch.Generator().manual_seed(1)
    lens = [37, 200, 16]
    NB = sum(-(-L // 16) for L in lens) + 3
    kp = torch.randn(NB, 4, 16, 64, generator=gen).to(cuda_device)
    vp = torch.randn(NB, 4, 16, 64, generator=gen).to(cuda_device)
    tables = random_tables(rng, lens, NB, 16)
    cache = build_cache(b2pa, kp, vp, tables, lens, 16)
    q = strided_q(3, 4, 1, 64, torch.float32, cuda_device, gen)
    out = b2pa.paged_attention("b200_paged", q, cache, 1)
    ref = orc.paged_attention_c(q.cpu().numpy(), kp.cpu().numpy(), vp.cpu().numpy(), tables, lens, [1, 1, 1])
    np.testing.assert_allclose(out.cpu().numpy(), ref, **TOL[torch.float32])
    assert b2pa.read_status(cuda_device) == 0
