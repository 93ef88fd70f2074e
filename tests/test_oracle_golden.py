"""Pins the CPU oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as orc
from tests._helpers import load_golden, split_tables

ATTN_CASES = [
    "decode_f32_bs8_d16",
    "decode_f32_curvar",
    "decode_f32_bs16_d64",
    "prefill_f32_bs16_d32",
    "prefill_f32_bs8_d16",
    "prefill_bf16_bs16_d64",
    "decode_bf16_bs16_d128",
]


def _f32(arr: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return (arr.astype(np.uint32) << 16).view(np.float32)
    return arr.astype(np.float32)


@pytest.mark.parametrize("name", ATTN_CASES)
@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_attention_oracle_matches_reference(name, impl):
    g = load_golden(name)
    dt = str(g["dtype"])
    q, kp, vp = _f32(g["q"], dt), _f32(g["k_pool"], dt), _f32(g["v_pool"], dt)
    tables = split_tables(g["block_ids"], g["block_counts"])
    fn = orc.paged_attention_np if impl == "numpy" else orc.paged_attention_c
    out = fn(q, kp, vp, tables, g["seq_lens"], [int(x) for x in g["cur_lens"]])
    np.testing.assert_allclose(out, g["out"], rtol=2e-5, atol=2e-6)


def test_c_oracle_strided_q_and_threads():
    g = load_golden("prefill_f32_bs16_d32")
    tables = split_tables(g["block_ids"], g["block_counts"])
    q = np.ascontiguousarray(g["q"].transpose(0, 2, 1, 3)).transpose(0, 2, 1, 3)  # [B,H,T,D] view of [B,T,H,D]
    assert not q.flags["C_CONTIGUOUS"]
    for nt in (1, 3):
        out = orc.paged_attention_c(q, g["k_pool"], g["v_pool"], tables, g["seq_lens"], list(g["cur_lens"]), nthreads=nt)
        np.testing.assert_allclose(out, g["out"], rtol=2e-5, atol=2e-6)


def test_allocator_and_append_oracle_matches_reference():
    g = load_golden("alloc_sequence")
    pool = orc.OraclePool(int(g["block_size"]), int(g["initial_blocks"]), float(g["growth_factor"]))
    states = [orc.OracleState(pool) for _ in range(3)]
    for i in range(int(g["n_steps"])):
        rel = int(g[f"step{i}_release"])
        if rel >= 0:
            states[rel].release()
        kind = str(g[f"step{i}_lens_kind"])
        lens = None if kind == "none" else (int(g[f"step{i}_lens"][0]) if kind == "int" else list(g[f"step{i}_lens"]))
        ret = orc.oracle_append_batch(states, g[f"step{i}_k"], g[f"step{i}_v"], lens)
        assert ret == g[f"step{i}_ret"].tolist()
        assert [b for s in states for b in s.block_ids] == g[f"step{i}_block_ids"].tolist()
        assert [len(s.block_ids) for s in states] == g[f"step{i}_block_counts"].tolist()
        assert pool.free == g[f"step{i}_free"].tolist()
        assert pool.capacity == int(g[f"step{i}_capacity"])
    assert np.array_equal(pool.k.view(np.uint32), g["k_pool"].view(np.uint32))
    assert np.array_equal(pool.v.view(np.uint32), g["v_pool"].view(np.uint32))


def test_bf16_round_matches_torch():
    import torch

    x = np.random.default_rng(0).standard_normal(4096).astype(np.float32) * 100
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(orc.bf16_round(x), ref)


def test_visible_count_rules():
    # decode: all keys; cur 0: all keys; cur 2 on a decode row: one fewer
    assert orc.visible_count(10, 1, 0) == 10
    assert orc.visible_count(10, 0, 0) == 10
    assert orc.visible_count(10, 2, 0) == 9
    # prefill padded row sees the whole sequence; first chunk row sees past+1
    assert orc.visible_count(20, 5, 7) == 20
    assert orc.visible_count(20, 5, 0) == 16
    assert orc.visible_count(0, 0, 0) == 0
    assert orc.visible_count(3, 5, 0) == 0


@pytest.mark.parametrize("name", ["decode_f32_curvar", "prefill_f32_bs8_d16", "decode_bf16_bs16_d128"])
def test_token_loop_restatement_matches_reference(name):
    """The per-token loop form bench.py times as the reference's CPU path
    computes the reference's outputs."""
    import torch

    from oracle import torch_paged as tp

    g = load_golden(name)
    dt = str(g["dtype"])
    q, kp, vp = _f32(g["q"], dt), _f32(g["k_pool"], dt), _f32(g["v_pool"], dt)
    tables = split_tables(g["block_ids"], g["block_counts"])
    kt, vt = torch.from_numpy(kp), torch.from_numpy(vp)
    for b in range(q.shape[0]):
        out = tp.paged_attention_token_loop(torch.from_numpy(q[b]), kt, vt, tables[b], int(g["seq_lens"][b]),
                                            int(g["cur_lens"][b]))
        np.testing.assert_allclose(out.numpy(), g["out"][b], rtol=2e-5, atol=2e-6)
