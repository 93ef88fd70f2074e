"""Pins the model restatement used by the end-to-end tests (oracle/model.py)
to the reference itself: same weights from set_seed(42) (state-dict digest),
same greedy tokens and logits on CPU with the torch restatement of the
reference's attention (oracle/torch_paged.py).  CPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import model as om
from tests._helpers import load_golden


def _tiny(backend, device="cpu"):
    om.set_seed(42)
    m = om.TinyLM(128, 64, 4, 2, 128, 128, backend, kv_block_size=8, kv_pool_initial_blocks=8,
                  kv_pool_growth_factor=2.0)
    prompt = torch.randint(0, 128, (2, 16))
    return m.to(device).eval(), prompt.to(device)


def test_tiny_model_matches_reference_on_cpu():
    g = load_golden("model_tiny")
    model, prompt = _tiny(om.torch_reference_backend())
    assert om.state_dict_digest(model) == bytes(g["weights_sha256"]).decode()
    assert np.array_equal(prompt.numpy(), g["prompt"])
    toks, logits, _ = om.generate_with_cache(model, prompt, 6, keep_logits=True)
    assert np.array_equal(toks.numpy(), g["tokens"])
    np.testing.assert_allclose(logits[0].numpy(), g["prefill_logits"], rtol=1e-5, atol=1e-5)


def test_config0_model_matches_reference_on_cpu():
    """BASELINE config[0] on CPU: weights, prompt, all 128 greedy tokens, the
    prefill and final logits, and the layer-0 block ids match the reference."""
    torch.set_num_threads(max(torch.get_num_threads(), 1))
    g = load_golden("model_config0")
    model, prompt = om.config0_model(om.torch_reference_backend(), "cpu")
    assert om.state_dict_digest(model) == bytes(g["weights_sha256"]).decode()
    assert np.array_equal(prompt.numpy(), g["prompt"])
    toks, logits, caches = om.generate_with_cache(model, prompt, 128, keep_logits=True)
    assert np.array_equal(toks.numpy(), g["tokens"])
    np.testing.assert_allclose(logits[0].numpy(), g["prefill_logits"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(logits[-1].numpy(), g["final_logits"], rtol=1e-4, atol=1e-5)
    st = caches[0] if not hasattr(caches[0], "states") else caches[0].states[0]
    assert st.block_ids == g["layer0_block_ids"].tolist()
    assert float(st.pool.k_blocks.double().sum()) == pytest.approx(float(g["layer0_k_pool_sum"]), rel=1e-6)
