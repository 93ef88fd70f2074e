"""One decode step of the reference's model on b2pa kernels only.

The reference's ``TinyTransformerLM`` (src/model/transformer.py:38-181) runs
a decode step as torch modules: embeddings, then per block LayerNorm, three
projections, paged attention, output projection, residual, LayerNorm, a
two-layer GELU MLP, residual (:7-35; src/model/attention.py:46-64), then the
final LayerNorm, lm_head and the greedy argmax
(src/inference/generate_with_cache.py:204).  With one new token per request
every product is a matrix-vector product, bound by reading the weights.
``FusedDecoder`` runs the same step as

    b2pa_rows_embed
    per block:  b2pa_rows_linear (LN1 + fused q/k/v projection)
                append_batch + paged_attention (one b2pa_paged_decode_append)
                b2pa_rows_linear (output projection + residual add)
                b2pa_rows_linear (LN2 + first MLP layer + GELU)
                b2pa_rows_linear (second MLP layer + residual add)
    b2pa_rows_linear (final LN + lm_head), b2pa_rows_argmax

-- four launches per block plus the attention, each weight matrix read once,
in buffers that stay at fixed addresses, so the whole step can be captured
by ``b2pa.DecodeGraph``.  It reads the model's parameters through the
reference's module names (token_emb, pos_emb, blocks[i].ln1 / attn.q_proj /
k_proj / v_proj / out_proj / ln2 / mlp[0] / mlp[2], ln_f, lm_head); the
q/k/v weights are concatenated once at construction, so build it again after
changing the model's weights.  fp32 models only (the reference's dtype).
"""
from __future__ import annotations

import torch

from . import _lib


def collect_parameters(model) -> dict:
    """The decode step's parameters of a TinyTransformerLM-shaped model, read
    through the reference's module names (src/model/transformer.py:7-18,
    38-181; src/model/attention.py:9-30): embeddings, per block the two
    LayerNorms, the q/k/v weights concatenated into one [3d, d] matrix, the
    output projection and the two MLP layers, then the final LayerNorm and
    lm_head."""
    layers = []
    for blk in model.blocks:
        att = blk.attn
        layers.append({
            "ln1": (blk.ln1.weight.detach(), blk.ln1.bias.detach(), float(blk.ln1.eps)),
            "w_qkv": torch.cat([att.q_proj.weight, att.k_proj.weight, att.v_proj.weight]).detach().contiguous(),
            "b_qkv": torch.cat([att.q_proj.bias, att.k_proj.bias, att.v_proj.bias]).detach().contiguous(),
            "w_o": att.out_proj.weight.detach(), "b_o": att.out_proj.bias.detach(),
            "ln2": (blk.ln2.weight.detach(), blk.ln2.bias.detach(), float(blk.ln2.eps)),
            "w1": blk.mlp[0].weight.detach(), "b1": blk.mlp[0].bias.detach(),
            "w2": blk.mlp[2].weight.detach(), "b2": blk.mlp[2].bias.detach(),
            "H": att.num_heads,
        })
    return {"tok": model.token_emb.weight.detach(), "pos": model.pos_emb.weight.detach(), "layers": layers,
            "ln_f": (model.ln_f.weight.detach(), model.ln_f.bias.detach(), float(model.ln_f.eps)),
            "w_head": model.lm_head.weight.detach(),
            "b_head": model.lm_head.bias.detach() if model.lm_head.bias is not None else None}


class FusedDecoder:
    """Decode steps of a TinyTransformerLM-shaped fp32 model, up to
    ``max_batch`` (<= 16) requests per step."""

    def __init__(self, model, max_batch: int = 16):
        if not 1 <= max_batch <= 16:
            raise ValueError("b2pa.FusedDecoder: max_batch must be between 1 and 16")
        w = model.lm_head.weight
        if w.dtype != torch.float32 or not w.is_cuda:
            raise TypeError("b2pa.FusedDecoder: the model must be fp32 on a CUDA device")
        self.device = w.device
        P = collect_parameters(model)
        self.tok, self.pos, self.layers = P["tok"], P["pos"], P["layers"]
        self.ln_f, self.w_head, self.b_head = P["ln_f"], P["w_head"], P["b_head"]
        self.d = self.tok.shape[1]
        self.vocab = self.w_head.shape[0]
        self.d_ff = self.layers[0]["w1"].shape[0] if self.layers else 0
        for t in [self.tok, self.pos, self.w_head] + [v for L in self.layers for v in L.values()
                                                       if isinstance(v, torch.Tensor)]:
            if not t.is_contiguous():
                raise ValueError("b2pa.FusedDecoder: model parameters must be contiguous")
        dev, mb = self.device, max_batch
        self.max_batch = mb
        self.x = torch.empty(mb, self.d, device=dev)
        self.qkv = torch.empty(mb, 3 * self.d, device=dev)
        self.hid = torch.empty(mb, max(self.d_ff, 4), device=dev)
        self.logits = torch.empty(mb, self.vocab, device=dev)
        self.next_ids = torch.empty(mb, dtype=torch.int64, device=dev)

    def _linear(self, x, M, K, ln, w, b, N, y, act=0, acc=0):
        lib = _lib.load()
        dev = self.device
        rc = lib.b2pa_rows_linear(x.data_ptr(), x.stride(0), M, K,
                                  ln[0].data_ptr() if ln else None, ln[1].data_ptr() if ln else None,
                                  ln[2] if ln else 0.0, w.data_ptr(), b.data_ptr() if b is not None else None, N,
                                  act, y.data_ptr(), y.stride(0), acc, _lib.status_buffer(dev).data_ptr(),
                                  _lib.stream_handle(dev))
        _lib.check(rc, "b2pa_rows_linear")

    def step(self, token_ids: torch.Tensor, positions: torch.Tensor, layer_caches) -> tuple[torch.Tensor, torch.Tensor]:
        """One decode token for each of the M requests: ``token_ids`` and
        ``positions`` are int64 device tensors [M]; ``layer_caches[l]`` is the
        batch object of layer l (``states`` + ``pool``: this package's
        BatchedPagedKVCache or the reference's).  Returns (logits [M, vocab],
        greedy ids [M]) -- views of this object's buffers, rewritten by the
        next step."""
        from .attention import paged_attention

        M = token_ids.shape[0]
        if M > self.max_batch:
            raise ValueError(f"b2pa.FusedDecoder: {M} requests exceed max_batch {self.max_batch}")
        lib = _lib.load()
        dev = self.device
        status = _lib.status_buffer(dev).data_ptr()
        d = self.d
        _lib.check(lib.b2pa_rows_embed(token_ids.data_ptr(), positions.data_ptr(), M, self.tok.data_ptr(),
                                       self.tok.shape[0], self.pos.data_ptr(), self.pos.shape[0], d,
                                       self.x.data_ptr(), self.x.stride(0), status, _lib.stream_handle(dev)),
                   "b2pa_rows_embed")
        for L, cache in zip(self.layers, layer_caches):
            H = L["H"]
            D = d // H
            self._linear(self.x, M, d, L["ln1"], L["w_qkv"], L["b_qkv"], 3 * d, self.qkv)
            # q, k, v as [M, H, 1, D] views of the fused projection's rows
            q, k, v = (self.qkv.as_strided((M, H, 1, D), (3 * d, D, D, 1), i * d) for i in range(3))
            cache.append_batch(k, v, 1)
            out = paged_attention("b200_paged", q, cache, 1)          # [M, H, 1, D], contiguous
            self._linear(out.reshape(M, d), M, d, None, L["w_o"], L["b_o"], d, self.x, acc=1)
            self._linear(self.x, M, d, L["ln2"], L["w1"], L["b1"], self.d_ff, self.hid, act=1)
            self._linear(self.hid, M, self.d_ff, None, L["w2"], L["b2"], d, self.x, acc=1)
        self._linear(self.x, M, d, self.ln_f, self.w_head, self.b_head, self.vocab, self.logits)
        _lib.check(lib.b2pa_rows_argmax(self.logits.data_ptr(), self.logits.stride(0), M, self.vocab,
                                        self.next_ids.data_ptr(), status, _lib.stream_handle(dev)),
                   "b2pa_rows_argmax")
        return self.logits[:M], self.next_ids[:M]


class FusedDecodeExecutor:
    """A decode executor with the contract of the reference's
    ``run_decode_step`` (src/serving/continuous_generate.py:198-276), for its
    ``ContinuousBatchingScheduler`` or ``b2pa.serve``: ``executor(requests,
    start_time_ms, event_id)`` advances every request by one greedy token and
    returns the reference's result dict.  The step runs on ``FusedDecoder``
    inside a ``DecodeStep`` (allocation for all layers at once, one shared
    block table), timed like the reference's (device synchronised on both
    sides, host work included).  The requests' KV caches must exist (their
    prompt was prefilled).  Per-request bookkeeping follows the reference:
    start time and batch id on first service, the new token appended, phase
    and finish time updated, completed requests returned."""

    def __init__(self, model, device, max_batch: int = 16):
        self.model = model
        self.device = torch.device(device)
        self.decoder = FusedDecoder(model, max_batch=max_batch)
        self.ids = torch.empty(max_batch, dtype=torch.int64, device=self.device)
        self.pos = torch.empty(max_batch, dtype=torch.int64, device=self.device)
        self.host = torch.empty(2, max_batch, dtype=torch.int64, pin_memory=True)
        self.meta = None

    @torch.no_grad()
    def __call__(self, requests: list, start_time_ms: float, event_id: int) -> dict:
        import time

        from .paged_kv import BatchedPagedKVCache
        from .step import DecodeStep

        if not requests:
            return {"batch_runtime_ms": 0.0, "requests_completed": []}
        M = len(requests)
        n_layers = len(self.decoder.layers)
        layer_states = [[r.kv_caches[l] for r in requests] for l in range(n_layers)]
        batches = [BatchedPagedKVCache(states=states, pool=states[0].pool) for states in layer_states]
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        h = self.host.numpy()
        h[0, :M] = [r.generated_token_ids[-1] for r in requests]
        h[1, :M] = [r.prompt_len + len(r.generated_token_ids) - 1 for r in requests]
        self.ids[:M].copy_(self.host[0, :M], non_blocking=True)
        self.pos[:M].copy_(self.host[1, :M], non_blocking=True)
        step = DecodeStep(layer_states, self.meta)
        with step:
            _, nxt = self.decoder.step(self.ids[:M], self.pos[:M], batches)
        self.meta = step.meta
        next_tokens = nxt.tolist()
        torch.cuda.synchronize(self.device)
        elapsed_ms = (time.perf_counter() - t0) * 1000.0
        finish_ms = start_time_ms + elapsed_ms
        completed = []
        for r, tok in zip(requests, next_tokens):
            if r.start_time_ms is None:
                r.start_time_ms = start_time_ms
                r.batch_id = event_id
            r.scheduler_mode = "continuous"
            r.generated_token_ids.append(int(tok))
            if len(r.generated_token_ids) >= r.max_new_tokens:
                r.phase = "finished"
                r.finish_time_ms = finish_ms
                completed.append(r)
            else:
                r.phase = "decode"
        return {"batch_runtime_ms": elapsed_ms, "requests_completed": completed, "batch_size": M,
                "tokens_scheduled": M, "phase": "decode", "prompt_len": max(r.prompt_len for r in requests),
                "max_new_tokens": max(r.max_new_tokens for r in requests), "prefill_tokens": 0, "decode_tokens": M,
                "decode_kernel_tokens": M, "prefill_runtime_ms": 0.0, "decode_runtime_ms": elapsed_ms,
                "decode_ms_per_token": elapsed_ms / M, "backend_name": "b200_paged_fused"}
