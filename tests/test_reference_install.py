"""b2pa against the reference's own objects, on the CPU.  Runs only where a
checkout of the reference is available (B2PA_REFERENCE_ROOT names its root;
it is never needed on the GPU box): the shim rebinds and restores the real
reference symbols and leaves its CPU path intact; the decode-step planner
allocates on the reference's own pools exactly what the reference's
append_batch allocates; the decoder finds its parameters under the real
model's module names; b2pa.serve with one rank takes the same decisions as
the reference's ContinuousBatchingScheduler."""
from __future__ import annotations

import copy
import importlib
import os
import sys

import pytest
import torch

import b2pa

REF = os.environ.get("B2PA_REFERENCE_ROOT")
pytestmark = pytest.mark.skipif(not REF, reason="B2PA_REFERENCE_ROOT is not set (no reference checkout here)")


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, REF)
    try:
        # the modules themselves (the packages re-export same-named functions)
        names = {"cache": "src.cache.paged_kv", "gen": "src.inference.generate_with_cache",
                 "kern": "src.kernels.paged_attention", "attn": "src.model.attention", "tr": "src.model.transformer",
                 "loadgen": "src.serving.loadgen", "sched": "src.serving.scheduler"}
        yield {k: importlib.import_module(v) for k, v in names.items()}
    finally:
        sys.path.remove(REF)


def _tiny(ref, backend):
    torch.manual_seed(0)
    return ref["tr"].TinyTransformerLM(vocab_size=128, d_model=64, num_heads=4, num_layers=2, d_ff=128,
                                       max_seq_len=128, attention_backend=backend, kv_block_size=8,
                                       kv_pool_initial_blocks=8, kv_pool_growth_factor=2.0).eval()


def test_install_rebinds_the_real_symbols_and_keeps_the_cpu_path(ref):
    kern, attn, cache = ref["kern"], ref["attn"], ref["cache"]
    orig_pa, orig_append = kern.paged_attention, cache.BatchedPagedKVCache.append_batch
    prompt = torch.randint(0, 128, (2, 16), generator=torch.Generator().manual_seed(1))
    base = ref["gen"].generate_with_cache(_tiny(ref, "paged_reference"), prompt, max_new_tokens=[3, 3])
    handle = b2pa.install_into_reference("src", fuse_append=True)
    try:
        assert kern.paged_attention is attn.paged_attention and kern.paged_attention is not orig_pa
        assert cache.BatchedPagedKVCache.append_batch is not orig_append
        # CPU tensors keep the reference's own path, through the rebound symbols
        got = ref["gen"].generate_with_cache(_tiny(ref, "triton_paged"), prompt, max_new_tokens=[3, 3])
        for a, b in zip(base["generated_ids"], got["generated_ids"]):
            assert torch.equal(a, b)
        pool = cache.LayerBlockPool(8, 8, 2.0)
        pool._b2pa_pending = None   # the attributes the deferred append and the decode step keep on a pool
        pool._b2pa_step = None
    finally:
        handle.uninstall()
    assert kern.paged_attention is orig_pa and attn.paged_attention is orig_pa
    assert cache.BatchedPagedKVCache.append_batch is orig_append


def test_lockstep_plan_on_the_reference_pools(ref):
    from b2pa.step import reserve_lockstep

    cache = ref["cache"]
    lens = [13, 16, 40]

    def layers():
        out, pools = [], []
        for _ in range(3):
            pool = cache.LayerBlockPool(16, 4, 2.0)
            states = [cache.PagedKVCacheState(pool=pool) for _ in lens]
            k = torch.randn(3, 2, 40, 8, generator=torch.Generator().manual_seed(2))
            cache.BatchedPagedKVCache(states=states, pool=pool).append_batch(k, k, torch.tensor(lens))
            out.append(states)
            pools.append(pool)
        return out, pools

    mine, my_pools = layers()
    theirs, their_pools = layers()
    for step in range(30):
        reserve_lockstep(mine, my_pools)
        one = torch.zeros(3, 2, 1, 8)
        for states, pool in zip(theirs, their_pools):
            cache.BatchedPagedKVCache(states=states, pool=pool).append_batch(one, one, 1)
        for a, b in zip(mine, theirs):
            assert [s.block_ids for s in a] == [s.block_ids for s in b]
            assert [s.seq_len for s in a] == [s.seq_len for s in b]
        assert [p.free_block_ids for p in my_pools] == [p.free_block_ids for p in their_pools]


def test_decoder_finds_the_real_model_parameters(ref):
    from b2pa.decoder import collect_parameters

    model = _tiny(ref, "paged_reference")
    P = collect_parameters(model)
    assert P["tok"].shape == (128, 64) and P["pos"].shape == (128, 64) and P["w_head"].shape == (128, 64)
    assert len(P["layers"]) == 2
    L = P["layers"][0]
    assert L["w_qkv"].shape == (192, 64) and L["b_qkv"].shape == (192,) and L["H"] == 4
    assert L["w1"].shape == (128, 64) and L["w2"].shape == (64, 128) and L["ln1"][2] == model.blocks[0].ln1.eps
    assert torch.equal(L["w_qkv"][64:128], model.blocks[0].attn.k_proj.weight)


def test_one_rank_serve_matches_the_reference_scheduler(ref):
    from oracle import serving as osv

    RequestWorkloadProfile = importlib.import_module("src.config").RequestWorkloadProfile
    profiles = [RequestWorkloadProfile(p.name, p.prompt_len_min, p.prompt_len_max, p.max_new_tokens_min,
                                       p.max_new_tokens_max, p.weight) for p in osv.CONFIG3_PROFILES]
    reqs = ref["loadgen"].generate_requests(200, 52.0, 5000, workload_profiles=profiles, seed=42)
    theirs = copy.deepcopy(reqs)
    done, events = ref["sched"].ContinuousBatchingScheduler(8, 256, 1536).run(
        theirs, osv.fake_prefill_executor, osv.fake_decode_executor)
    res = b2pa.serve(reqs, osv.fake_prefill_executor, osv.fake_decode_executor, max_batch_size=8,
                     prefill_chunk_size=256, max_tokens_per_iteration=1536)
    assert [(e["phase"], e["batch_size"], e["tokens_scheduled"]) for e in events] == \
        [(e["phase"], len(e["request_ids"]), e["tokens_scheduled"]) for e in res.events]
    assert [e["dispatch_time_ms"] for e in events] == [e["dispatch_time_ms"] for e in res.events]
    assert [(r.request_id, r.first_token_time_ms, r.finish_time_ms) for r in done] == \
        [(r.request_id, r.first_token_time_ms, r.finish_time_ms) for r in res.completed]
