"""Restatement of the reference's decoder-only model and cached greedy
generation -- TEST INFRASTRUCTURE ONLY (used by tests/ for the end-to-end
BASELINE config[0] and serving config[3] checks).

The reference model is the caller of the attention path, not the path, and
the reference cannot travel to the GPU box, so the tests drive the b2pa
backend through this restatement of
  src/model/transformer.py:7-181 (TinyTransformerLM, TransformerBlock),
  src/model/attention.py:9-78 (CausalSelfAttention),
  src/inference/generate_with_cache.py:113-260 (generate_with_cache).
Modules are created in the reference's order with the reference's shapes, so
``set_seed(42)`` gives bit-identical weights (pinned by
tests/test_model_harness.py against a hash of the reference's state dict).

The attention backend is pluggable: a ``backend`` object supplies the pool,
state and batch classes and the attention function -- b2pa's, or the torch
restatement of the reference's (oracle/torch_paged.py).
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn as nn


@dataclass
class Backend:
    name: str
    pool_cls: type
    state_cls: type
    batch_cls: type
    attention: callable  # (q, kv_cache, current_lengths) -> out


def b2pa_backend():
    import b2pa

    return Backend("b200_paged", b2pa.LayerBlockPool, b2pa.PagedKVCacheState, b2pa.BatchedPagedKVCache,
                   lambda q, kv, cur: b2pa.paged_attention("b200_paged", q, kv, cur))


def torch_reference_backend():
    from oracle import torch_paged as tp

    return Backend("torch_reference", tp.TorchBlockPool, tp.TorchCacheState, tp.TorchBatchedCache,
                   tp.paged_attention_torch)


def set_seed(seed: int) -> None:
    """src/utils/seed.py:6-11."""
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


class Attention(nn.Module):
    def __init__(self, d_model: int, num_heads: int, backend: Backend):
        super().__init__()
        self.d_model, self.num_heads, self.head_dim = d_model, num_heads, d_model // num_heads
        self.backend = backend
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)
        self.dropout = nn.Dropout(0.0)

    def _split(self, x):
        B, T, _ = x.shape
        return x.view(B, T, self.num_heads, self.head_dim).transpose(1, 2)

    def forward(self, x, kv_cache, current_lengths):
        q = self._split(self.q_proj(x))
        k = self._split(self.k_proj(x))
        v = self._split(self.v_proj(x))
        if isinstance(kv_cache, self.backend.state_cls):
            kv_cache = self.backend.batch_cls(states=[kv_cache], pool=kv_cache.pool)
        kv_cache.append_batch(k, v, current_lengths=current_lengths)
        out = self.backend.attention(q, kv_cache, current_lengths)
        B, _, T, _ = out.shape
        out = self.out_proj(out.transpose(1, 2).contiguous().view(B, T, self.d_model))
        return out, (kv_cache.states[0] if len(kv_cache.states) == 1 else kv_cache)


class Block(nn.Module):
    def __init__(self, d_model, num_heads, d_ff, backend):
        super().__init__()
        self.ln1 = nn.LayerNorm(d_model)
        self.attn = Attention(d_model, num_heads, backend)
        self.ln2 = nn.LayerNorm(d_model)
        self.mlp = nn.Sequential(nn.Linear(d_model, d_ff), nn.GELU(), nn.Linear(d_ff, d_model), nn.Dropout(0.0))

    def forward(self, x, kv_cache, current_lengths):
        a, kv_cache = self.attn(self.ln1(x), kv_cache, current_lengths)
        x = x + a
        x = x + self.mlp(self.ln2(x))
        return x, kv_cache


class TinyLM(nn.Module):
    """TinyTransformerLM (src/model/transformer.py:38-181), cached path only."""

    def __init__(self, vocab_size, d_model, num_heads, num_layers, d_ff, max_seq_len, backend: Backend,
                 kv_block_size=16, kv_pool_initial_blocks=64, kv_pool_growth_factor=2.0):
        super().__init__()
        self.backend = backend
        self.kv_block_size = kv_block_size
        self.kv_pool_initial_blocks = kv_pool_initial_blocks
        self.kv_pool_growth_factor = kv_pool_growth_factor
        self.token_emb = nn.Embedding(vocab_size, d_model)
        self.pos_emb = nn.Embedding(max_seq_len, d_model)
        self.blocks = nn.ModuleList([Block(d_model, num_heads, d_ff, backend) for _ in range(num_layers)])
        self.ln_f = nn.LayerNorm(d_model)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        self.pools = None

    def _pools(self):
        if self.pools is None:
            self.pools = [self.backend.pool_cls(self.kv_block_size, self.kv_pool_initial_blocks,
                                                self.kv_pool_growth_factor) for _ in self.blocks]
        return self.pools

    def create_request_kv_caches(self, batch_size: int):
        pools = self._pools()
        return [[self.backend.state_cls(pool=pools[i]) for i in range(len(self.blocks))] for _ in range(batch_size)]

    def forward(self, input_ids, kv_caches=None, position_offset=0, current_lengths=None):
        B, T = input_ids.shape
        dev = input_ids.device
        if isinstance(position_offset, int):
            pos = torch.arange(position_offset, position_offset + T, device=dev).unsqueeze(0).expand(B, T)
        else:
            pos = position_offset.view(B, 1) + torch.arange(T, device=dev).view(1, T)
        x = self.token_emb(input_ids) + self.pos_emb(pos)
        if kv_caches is None:
            per_req = self.create_request_kv_caches(B)
            if B > 1:
                pools = self._pools()
                kv_caches = [self.backend.batch_cls(states=[per_req[r][i] for r in range(B)], pool=pools[i])
                             for i in range(len(self.blocks))]
            else:
                kv_caches = [per_req[0][i] for i in range(len(self.blocks))]
        new = []
        for i, blk in enumerate(self.blocks):
            x, c = blk(x, kv_caches[i], current_lengths)
            new.append(c)
        return self.lm_head(self.ln_f(x)), new


def state_dict_digest(model: nn.Module) -> str:
    import hashlib

    h = hashlib.sha256()
    for name, t in model.state_dict().items():
        h.update(name.encode())
        h.update(t.detach().cpu().contiguous().numpy().tobytes())
    return h.hexdigest()


@torch.no_grad()
def generate_with_cache(model: TinyLM, prompt_ids: torch.Tensor, max_new_tokens: int, keep_logits: bool = False):
    """Greedy cached generation for a batch of equal-length prompts, following
    src/inference/generate_with_cache.py:142-215: prefill with
    current_lengths = prompt lengths, then one-token decode steps with
    position_offset = prompt_len + generated - 1 and current_lengths = 1.
    Returns (tokens [B, max_new_tokens], per-step logits or None, kv_caches)."""
    B, P = prompt_ids.shape
    dev = prompt_ids.device
    lengths = torch.full((B,), P, dtype=torch.long, device=dev)
    logits, caches = model(prompt_ids, position_offset=0, current_lengths=lengths)
    step_logits = [logits[:, P - 1, :].float().cpu()] if keep_logits else None
    nxt = torch.argmax(logits[torch.arange(B, device=dev), lengths - 1, :], dim=-1)
    tokens = [nxt.cpu()]
    if B > 1:
        batched = caches
    else:
        batched = caches
    for step in range(1, max_new_tokens):
        pos = torch.full((B,), P + step - 1, dtype=torch.long, device=dev)
        if B > 1:
            batched = [model.backend.batch_cls(states=list(c.states), pool=c.pool) for c in batched]
        logits, batched = model(nxt.view(B, 1), kv_caches=batched, position_offset=pos, current_lengths=1)
        if keep_logits:
            step_logits.append(logits[:, -1, :].float().cpu())
        nxt = torch.argmax(logits[:, -1, :], dim=-1)
        tokens.append(nxt.cpu())
    return torch.stack(tokens, dim=1), step_logits, batched


def config0_model(backend: Backend, device) -> tuple[TinyLM, torch.Tensor]:
    """set_seed(42); TinyTransformerLM(5000, 512, 8, 6,
    2048, 1024, block 16) built on CPU then moved; prompt randint(0, 5000,
    (1, 128)) drawn after the model."""
    set_seed(42)
    model = TinyLM(5000, 512, 8, 6, 2048, 1024, backend, kv_block_size=16, kv_pool_initial_blocks=64,
                   kv_pool_growth_factor=2.0)
    prompt = torch.randint(0, 5000, (1, 128))
    return model.to(device).eval(), prompt.to(device)
