"""Generates the golden vectors in tests/golden/*.npz by running the
reference implementation itself (jacobzhang22/efficient-inference-system).

Run here, where the reference checkout is available (read-only):

    python tests/golden/make_golden.py --reference /path/to/reference

Every case drives the reference's own public API on CPU:
``LayerBlockPool`` / ``PagedKVCacheState`` / ``BatchedPagedKVCache.append_batch``
(src/cache/paged_kv.py) for pools and block tables, and
``paged_attention_reference`` (src/kernels/reference_paged_attention.py) for
attention outputs.  The fixtures are small and committed; the GPU box never
needs the reference.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

OUT_DIR = Path(__file__).resolve().parent


def _import_reference(path: str):
    sys.path.insert(0, path)
    from src.cache.paged_kv import BatchedPagedKVCache, LayerBlockPool, PagedKVCacheState
    from src.kernels.reference_paged_attention import paged_attention_reference
    return BatchedPagedKVCache, LayerBlockPool, PagedKVCacheState, paged_attention_reference


def _tables(states) -> tuple[np.ndarray, np.ndarray]:
    flat = np.array([b for s in states for b in s.block_ids], dtype=np.int32)
    counts = np.array([len(s.block_ids) for s in states], dtype=np.int32)
    return flat, counts


def case_alloc_sequence(ref) -> dict:
    """Allocator growth, block-boundary appends, clamping, release + LIFO reuse."""
    Batched, Pool, State, _ = ref
    torch.manual_seed(1)
    pool = Pool(block_size=4, initial_blocks=2, growth_factor=2.0)
    states = [State(pool=pool) for _ in range(3)]
    cache = Batched(states=states, pool=pool)
    H, D = 2, 8
    steps = [
        (6, torch.tensor([6, 1, 0]), None),
        (1, None, None),
        (5, [5, 4, 3], 1),          # release state 1 before this append
        (3, 7, None),               # int length larger than T: clamped to T
        (4, torch.tensor([0, 4, 2]), None),
    ]
    rec: dict = {"H": H, "D": D, "block_size": 4, "initial_blocks": 2, "growth_factor": 2.0,
                 "n_steps": len(steps)}
    for i, (T, lens, release_idx) in enumerate(steps):
        if release_idx is not None:
            states[release_idx].release()
        k = torch.randn(3, H, T, D)
        v = torch.randn(3, H, T, D)
        if isinstance(lens, list):
            lens_arg = torch.tensor(lens)
        else:
            lens_arg = lens
        ret = cache.append_batch(k, v, current_lengths=lens_arg)
        flat, counts = _tables(states)
        rec[f"step{i}_T"] = T
        rec[f"step{i}_lens_kind"] = "none" if lens is None else ("int" if isinstance(lens, int) else "list")
        rec[f"step{i}_lens"] = np.array([0, 0, 0] if lens is None else ([lens] * 3 if isinstance(lens, int) else
                                        [int(x) for x in (lens.tolist() if torch.is_tensor(lens) else lens)]),
                                        dtype=np.int64)
        rec[f"step{i}_release"] = -1 if release_idx is None else release_idx
        rec[f"step{i}_k"] = k.numpy()
        rec[f"step{i}_v"] = v.numpy()
        rec[f"step{i}_ret"] = ret.numpy()
        rec[f"step{i}_block_ids"] = flat
        rec[f"step{i}_block_counts"] = counts
        rec[f"step{i}_free"] = np.array(pool.free_block_ids, dtype=np.int32)
        rec[f"step{i}_capacity"] = pool.capacity_blocks
    rec["k_pool"] = pool.k_blocks.numpy()
    rec["v_pool"] = pool.v_blocks.numpy()
    return rec


def _attention_case(ref, *, seed, B, H, D, bs, initial_blocks, prefix, T, cur, dtype=torch.float32) -> dict:
    """Prefix append, chunk append, then paged_attention_reference."""
    Batched, Pool, State, attn = ref
    torch.manual_seed(seed)
    pool = Pool(block_size=bs, initial_blocks=initial_blocks, growth_factor=2.0)
    states = [State(pool=pool) for _ in range(B)]
    cache = Batched(states=states, pool=pool)
    Tp = max(max(prefix), 1)
    kp = torch.randn(B, H, Tp, D).to(dtype)
    vp = torch.randn(B, H, Tp, D).to(dtype)
    cache.append_batch(kp, vp, current_lengths=torch.tensor(prefix))
    kc = torch.randn(B, H, T, D).to(dtype)
    vc = torch.randn(B, H, T, D).to(dtype)
    q = torch.randn(B, H, T, D).to(dtype)
    cur_t = torch.tensor(cur)
    cache.append_batch(kc, vc, current_lengths=cur_t)
    flat, counts = _tables(states)
    seq_lens = np.array([s.seq_len for s in states], dtype=np.int32)
    if dtype == torch.float32:
        out = attn(q=q, kv_cache=cache, current_lengths=cur_t)
        pool_k, pool_v, q_np = pool.k_blocks.numpy(), pool.v_blocks.numpy(), q.numpy()
    else:
        # bf16: the reference computes on the same bf16 values upcast to fp32.
        kb, vb = pool.k_blocks, pool.v_blocks
        pool.k_blocks, pool.v_blocks = kb.float(), vb.float()
        out = attn(q=q.float(), kv_cache=cache, current_lengths=cur_t)
        pool.k_blocks, pool.v_blocks = kb, vb
        pool_k = kb.view(torch.int16).numpy().view(np.uint16)
        pool_v = vb.view(torch.int16).numpy().view(np.uint16)
        q_np = q.view(torch.int16).numpy().view(np.uint16)
        kc = kc.float()
    return {
        "B": B, "H": H, "D": D, "block_size": bs, "T": T, "dtype": str(dtype).replace("torch.", ""),
        "prefix": np.array(prefix, dtype=np.int32), "cur_lens": np.array(cur, dtype=np.int32),
        "seq_lens": seq_lens, "block_ids": flat, "block_counts": counts,
        "k_pool": pool_k, "v_pool": pool_v, "q": q_np, "out": out.float().numpy(),
        "k_chunk": kc.numpy() if dtype == torch.float32 else kc.numpy(),
    }


def _model_case(ref_path: str, *, tiny: bool) -> dict:
    """Greedy cached generation by the reference itself on CPU with its torch
    paged attention (backend "paged_reference"): BASELINE config[0], or the
    reference's own test model (tests/test_paged_attention.py:10-38)."""
    import hashlib

    from src.inference.generate_with_cache import generate_with_cache
    from src.model.transformer import TinyTransformerLM
    from src.utils.seed import set_seed

    set_seed(42)
    if tiny:
        model = TinyTransformerLM(128, 64, 4, 2, 128, 128, attention_backend="paged_reference", kv_block_size=8,
                                  kv_pool_initial_blocks=8, kv_pool_growth_factor=2.0)
        prompt = torch.randint(0, 128, (2, 16))
        new_tokens = 6
    else:
        model = TinyTransformerLM(5000, 512, 8, 6, 2048, 1024, attention_backend="paged_reference",
                                  kv_block_size=16, kv_pool_initial_blocks=64, kv_pool_growth_factor=2.0)
        prompt = torch.randint(0, 5000, (1, 128))
        new_tokens = 128
    model.eval()
    h = hashlib.sha256()
    for name, t in model.state_dict().items():
        h.update(name.encode())
        h.update(t.detach().contiguous().numpy().tobytes())
    seen = []
    hook = model.lm_head.register_forward_hook(lambda m, i, o: seen.append(o.detach()[:, -1, :].clone()))
    res = generate_with_cache(model, prompt, max_new_tokens=new_tokens)
    hook.remove()
    gen = torch.stack([ids[prompt.shape[1]:] for ids in res["generated_ids"]])
    last = torch.stack(seen)                       # [steps, B, vocab] logits at the last position
    top2 = torch.topk(last, 2, dim=-1).values
    margins = (top2[..., 0] - top2[..., 1]).numpy()
    # the KV pool of layer 0 after generation, as a digest (the pools are large)
    caches = res["kv_caches"]
    k0 = caches[0].pool.k_blocks.contiguous().numpy()
    return {
        "weights_sha256": np.frombuffer(h.hexdigest().encode(), dtype=np.uint8),
        "prompt": prompt.numpy(), "tokens": gen.numpy(),
        "prefill_logits": last[0].numpy(), "final_logits": last[-1].numpy(),
        "margins": margins, "layer0_k_pool_sum": np.float64(k0.astype(np.float64).sum()),
        "layer0_block_ids": np.array(caches[0].states[0].block_ids, dtype=np.int32),
    }


def _serving_case() -> dict:
    """BASELINE config[3] request stream from the reference's load generator,
    and the reference's ContinuousBatchingScheduler(8, 256, 1536) run with the
    deterministic fake executors of oracle/serving.py (no model): pins the
    load generator and the scheduling policy."""
    sys.path.insert(0, str(OUT_DIR.parent.parent))
    from oracle import serving as osv
    from src.config import RequestWorkloadProfile
    from src.serving.loadgen import generate_requests
    from src.serving.metrics import percentile
    from src.serving.scheduler import ContinuousBatchingScheduler

    profiles = [RequestWorkloadProfile(p.name, p.prompt_len_min, p.prompt_len_max, p.max_new_tokens_min,
                                       p.max_new_tokens_max, p.weight) for p in osv.CONFIG3_PROFILES]
    reqs = generate_requests(200, 52.0, 5000, workload_profiles=profiles, seed=42)
    rec = {
        "arrival_ms": np.array([r.arrival_time_ms for r in reqs]),
        "prompt_len": np.array([r.prompt_len for r in reqs], dtype=np.int64),
        "max_new_tokens": np.array([r.max_new_tokens for r in reqs], dtype=np.int64),
        "prompt_id_sums": np.array([int(r.prompt_ids.sum()) for r in reqs], dtype=np.int64),
        "first_prompt": reqs[0].prompt_ids.numpy(),
        "workload": np.array([r.workload_name for r in reqs]),
    }
    sched = ContinuousBatchingScheduler(max_batch_size=8, prefill_chunk_size=256, max_tokens_per_iteration=1536)
    done, events = sched.run(reqs, prefill_executor=osv.fake_prefill_executor,
                             decode_executor=osv.fake_decode_executor)
    rec["ev_phase"] = np.array([e["phase"] for e in events])
    rec["ev_batch_size"] = np.array([e["batch_size"] for e in events], dtype=np.int64)
    rec["ev_dispatch_ms"] = np.array([e["dispatch_time_ms"] for e in events])
    rec["ev_tokens"] = np.array([e["tokens_scheduled"] for e in events], dtype=np.int64)
    rec["first_token_ms"] = np.array([r.first_token_time_ms for r in done])
    rec["finish_ms"] = np.array([r.finish_time_ms for r in done])
    ttft = [r.first_token_latency_ms for r in done if r.first_token_time_ms is not None]
    rec["ttft_p50_p99"] = np.array([percentile(ttft, 50), percentile(ttft, 99)])
    return rec


CASES = {
    "alloc_sequence": case_alloc_sequence,
    "decode_f32_bs8_d16": lambda ref: _attention_case(ref, seed=2, B=4, H=2, D=16, bs=8, initial_blocks=4,
                                                      prefix=[0, 7, 8, 23], T=1, cur=[1, 1, 1, 1]),
    "decode_f32_curvar": lambda ref: _attention_case(ref, seed=3, B=4, H=2, D=32, bs=16, initial_blocks=4,
                                                     prefix=[0, 15, 16, 40], T=1, cur=[1, 0, 2, 1]),
    "decode_f32_bs16_d64": lambda ref: _attention_case(ref, seed=4, B=2, H=4, D=64, bs=16, initial_blocks=8,
                                                       prefix=[128, 199], T=1, cur=[1, 1]),
    "prefill_f32_bs16_d32": lambda ref: _attention_case(ref, seed=5, B=3, H=2, D=32, bs=16, initial_blocks=4,
                                                        prefix=[0, 5, 20], T=12, cur=[12, 7, 0]),
    "prefill_f32_bs8_d16": lambda ref: _attention_case(ref, seed=6, B=2, H=4, D=16, bs=8, initial_blocks=8,
                                                       prefix=[3, 17], T=24, cur=[24, 9]),
    "prefill_bf16_bs16_d64": lambda ref: _attention_case(ref, seed=7, B=2, H=2, D=64, bs=16, initial_blocks=8,
                                                         prefix=[10, 40], T=20, cur=[20, 13],
                                                         dtype=torch.bfloat16),
    "decode_bf16_bs16_d128": lambda ref: _attention_case(ref, seed=8, B=3, H=2, D=128, bs=16, initial_blocks=8,
                                                         prefix=[1, 31, 64], T=1, cur=[1, 1, 1],
                                                         dtype=torch.bfloat16),
    "model_tiny": lambda ref: _model_case(REF_PATH[0], tiny=True),
    "model_config0": lambda ref: _model_case(REF_PATH[0], tiny=False),
    "serving_config3": lambda ref: _serving_case(),
}
REF_PATH = [None]  # the reference checkout, from --reference


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of a checkout of the reference repository")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    torch.set_num_threads(1)
    REF_PATH[0] = args.reference
    ref = _import_reference(args.reference)
    for name, fn in CASES.items():
        if args.only and name != args.only:
            continue
        rec = fn(ref)
        path = OUT_DIR / f"{name}.npz"
        np.savez_compressed(path, **{k: np.asarray(v) for k, v in rec.items()})
        print(f"wrote {path} ({path.stat().st_size} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
