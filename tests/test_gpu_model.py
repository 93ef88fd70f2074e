"""End-to-end model checks on the GPU (BASELINE config[0] and the reference's
own small-model test, tests/test_paged_attention.py:57-66 of the reference):
the model restatement (oracle/model.py, pinned to the reference on CPU) runs
once with the b2pa backend and once with the torch restatement of the
reference's attention on the same GPU.

* greedy tokens: identical between the two runs, and identical to the
  reference's own CPU run (golden; the smallest top-1/top-2 logit gap over
  the 128 steps is 1.2e-3, far above fp32 noise);
* logits at every step: rtol 1e-4 / atol 1e-5;
* KV pools: every append the b2pa run made is replayed through the torch
  restatement of the reference's append; pools and block tables must be
  bit-identical (and layer 0, whose inputs do not depend on attention, is
  bit-identical across the two runs).
"""
from __future__ import annotations

import json
import time

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import torch_paged as tp
from tests._helpers import load_golden

pytestmark = pytest.mark.gpu


class _Recorder:
    """Wraps a backend's batch class to record every append_batch call."""

    def __init__(self, backend):
        self.calls = []  # (layer pool id, [state index...], k, v, current_lengths)
        rec = self
        base = backend.batch_cls

        class Batch(base):
            def append_batch(self, k_new, v_new, current_lengths=None):
                rec.calls.append((id(self.pool), [id(s) for s in self.states], k_new.detach().clone(),
                                  v_new.detach().clone(),
                                  current_lengths.clone() if torch.is_tensor(current_lengths) else current_lengths))
                return super().append_batch(k_new, v_new, current_lengths)

        self.backend = om.Backend(backend.name, backend.pool_cls, backend.state_cls, Batch, backend.attention)


def _replay_pools(calls, pools, block_size, initial, growth):
    """Re-applies the recorded appends with the torch restatement of the
    reference's append; returns {pool id: TorchBlockPool} and state tables."""
    out = {id(p): tp.TorchBlockPool(block_size, initial, growth) for p in pools}
    states = {}
    for pool_id, sids, k, v, cur in calls:
        sts = [states.setdefault(s, tp.TorchCacheState(pool=out[pool_id])) for s in sids]
        tp.TorchBatchedCache(sts, pool=out[pool_id]).append_batch(k, v, cur)
    return out, states


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int32).numpy()


def _run(model, prompt, n):
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    toks, logits, caches = om.generate_with_cache(model, prompt, n, keep_logits=True)
    torch.cuda.synchronize()
    return toks, logits, caches, time.perf_counter() - t0


@pytest.mark.parametrize("fused", [False, True], ids=["append_then_decode", "fused_append"])
def test_config0_end_to_end(cuda_device, fused):
    """``fused``: decode-step appends deferred into the decode launch
    (b2pa.set_fused_append)."""
    import b2pa

    assert not torch.backends.cuda.matmul.allow_tf32
    g = load_golden("model_config0")
    rec = _Recorder(om.b2pa_backend())
    model_b, prompt = om.config0_model(rec.backend, cuda_device)
    model_r, prompt_r = om.config0_model(om.torch_reference_backend(), cuda_device)
    assert om.state_dict_digest(model_b) == bytes(g["weights_sha256"]).decode()
    assert torch.equal(prompt, prompt_r)
    prev = b2pa.set_fused_append(fused)
    try:
        om.generate_with_cache(model_b, prompt, 2)  # warm-up (library load, workspace, first launches)
        model_b.pools = None
        rec.calls.clear()
        toks_b, logits_b, caches_b, secs_b = _run(model_b, prompt, 128)
    finally:
        b2pa.set_fused_append(prev)
    toks_r, logits_r, caches_r, secs_r = _run(model_r, prompt, 128)
    assert torch.equal(toks_b, toks_r)
    assert np.array_equal(toks_b.numpy(), g["tokens"])
    for lb, lr in zip(logits_b, logits_r):
        np.testing.assert_allclose(lb.numpy(), lr.numpy(), rtol=1e-4, atol=1e-5)
    # pools: replay the recorded appends through the reference's append
    replay, rstates = _replay_pools(rec.calls, model_b.pools, 16, 64, 2.0)
    for pool in model_b.pools:
        ref_pool = replay[id(pool)]
        assert pool.capacity_blocks == ref_pool.capacity_blocks
        assert pool.free_block_ids == ref_pool.free_block_ids
        assert np.array_equal(_bits(pool.k_blocks), _bits(ref_pool.k_blocks))
        assert np.array_equal(_bits(pool.v_blocks), _bits(ref_pool.v_blocks))
    st_b = caches_b[0] if not hasattr(caches_b[0], "states") else caches_b[0].states[0]
    assert st_b.block_ids == g["layer0_block_ids"].tolist()
    # layer 0 inputs do not depend on attention: identical across the two backends
    assert np.array_equal(_bits(model_b.pools[0].k_blocks), _bits(model_r.pools[0].k_blocks))
    assert b2pa.read_status(cuda_device) == 0
    report = {"config": "BASELINE config[0]: 128-token prompt + 128 greedy tokens, batch 1, FP32",
              "decode_append": "fused into the decode launch" if fused else "separate append kernel",
              "b2pa_seconds": secs_b, "b2pa_tokens_per_s": 128 / secs_b,
              "torch_reference_on_gpu_seconds": secs_r}
    print(json.dumps(report))


@pytest.mark.parametrize("fused", [False, True], ids=["append_then_decode", "fused_append"])
def test_reference_small_model_tokens(cuda_device, fused):
    """The reference's own cross-backend check (tests/test_paged_attention.py:
    57-66): a 2-layer, 4-head, block-8 model, prompt (2, 16); greedy tokens of
    the GPU backend equal the torch reference path's and the reference's CPU
    run."""
    import b2pa

    g = load_golden("model_tiny")

    def tiny(backend):
        om.set_seed(42)
        m = om.TinyLM(128, 64, 4, 2, 128, 128, backend, kv_block_size=8, kv_pool_initial_blocks=8,
                      kv_pool_growth_factor=2.0)
        p = torch.randint(0, 128, (2, 16))
        return m.to(cuda_device).eval(), p.to(cuda_device)

    mb, pb = tiny(om.b2pa_backend())
    mr, pr = tiny(om.torch_reference_backend())
    prev = b2pa.set_fused_append(fused)
    try:
        tb, lb, _ = om.generate_with_cache(mb, pb, 6, keep_logits=True)
    finally:
        b2pa.set_fused_append(prev)
    tr, lr, _ = om.generate_with_cache(mr, pr, 6, keep_logits=True)
    assert torch.equal(tb, tr)
    assert np.array_equal(tb.numpy(), g["tokens"])
    for x, y in zip(lb, lr):
        np.testing.assert_allclose(x.numpy(), y.numpy(), rtol=1e-4, atol=1e-5)
