"""Paged attention entry points (decode and chunked prefill).

Mirrors the reference's backend call surface:

* ``paged_attention(backend, q, kv_cache, current_lengths)`` --
  src/kernels/paged_attention.py:13-51: validates the backend name, builds the
  block table and lengths on the device, and dispatches on ``q.shape[2] == 1``
  to decode, else to chunked prefill;
* ``paged_attention_decode_b200`` / ``paged_attention_prefill_b200`` -- the
  launchers, same arguments as ``paged_attention_decode_triton`` /
  ``paged_attention_prefill_triton`` (src/kernels/triton_paged_attention.py:
  179-258), returning ``torch.empty_like(q)`` filled by the CUDA kernels.

Every path runs the sm_100a kernels of libb2pa.so.  CPU tensors raise: this
package has no CPU or torch fallback.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._metadata import block_table_and_lengths
from .paged_kv import _kv_append, flush_pending, take_pending
from .step import _StepPending

# "triton_paged" is accepted so that models configured for the reference's GPU
# backend (src/model/transformer.py:55,117) run unchanged on this one.
SUPPORTED_BACKENDS = frozenset({"b200_paged", "triton_paged"})


def _attn_call(fn_name: str, q, k_pool, v_pool, page_table, seq_lens, current_lengths, max_pages: int | None = None):
    for t, name in ((q, "q"), (k_pool, "k_pool"), (v_pool, "v_pool")):
        if not t.is_cuda:
            raise RuntimeError(f"b2pa: {name} must be a CUDA tensor (this package has no CPU path)")
    if k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise TypeError(f"pool dtype {k_pool.dtype} differs from q dtype {q.dtype}")
    B, H, T, D = q.shape
    block_size = k_pool.shape[2]
    out = torch.empty_like(q)
    if max_pages is None:
        max_pages = page_table.shape[1]
    if page_table.numel() and page_table.stride(1) != 1:
        page_table = page_table.contiguous()
    pt_stride = page_table.stride(0) if page_table.dim() == 2 and page_table.numel() else max(max_pages, 1)
    seq_lens = seq_lens.to(dtype=torch.int32)
    cur = current_lengths.to(dtype=torch.int32)
    dev = q.device
    dt = _lib.dtype_code(q.dtype)
    lib = _lib.load()
    scale = 1.0 / math.sqrt(D)
    common_tail = (_lib.status_buffer(dev).data_ptr(), _lib.stream_handle(dev))
    if fn_name == "decode":
        ws_bytes = lib.b2pa_paged_decode_workspace_size(B, H, D, max_pages, block_size, dt)
        ws = _lib.workspace(dev, ws_bytes) if ws_bytes else None
        rc = lib.b2pa_paged_decode(
            q.data_ptr(), _lib.strides4(q), k_pool.data_ptr(), v_pool.data_ptr(), _lib.strides4(k_pool),
            k_pool.shape[0], page_table.data_ptr() if max_pages else None, pt_stride, max_pages,
            seq_lens.data_ptr(), cur.data_ptr(), out.data_ptr(), _lib.strides4(out),
            B, H, D, block_size, scale, dt,
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, *common_tail)
        _lib.check(rc, "b2pa_paged_decode")
    else:
        ws_bytes = lib.b2pa_paged_prefill_workspace_size(B, H, T, D, max_pages, block_size, dt)
        ws = _lib.workspace(dev, ws_bytes) if ws_bytes else None
        rc = lib.b2pa_paged_prefill(
            q.data_ptr(), _lib.strides4(q), k_pool.data_ptr(), v_pool.data_ptr(), _lib.strides4(k_pool),
            k_pool.shape[0], page_table.data_ptr() if max_pages else None, pt_stride, max_pages,
            seq_lens.data_ptr(), cur.data_ptr(), out.data_ptr(), _lib.strides4(out),
            B, H, T, D, block_size, scale, dt,
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, *common_tail)
        _lib.check(rc, "b2pa_paged_prefill")
    return out


def paged_attention_decode_b200(q, k_pool, v_pool, page_table, seq_lens, current_lengths) -> torch.Tensor:
    """Single-query paged attention (T == 1); replaces
    paged_attention_decode_triton (src/kernels/triton_paged_attention.py:179)."""
    return _attn_call("decode", q, k_pool, v_pool, page_table, seq_lens, current_lengths)


def paged_attention_prefill_b200(q, k_pool, v_pool, page_table, seq_lens, current_lengths) -> torch.Tensor:
    """Chunked-prefill paged attention; replaces paged_attention_prefill_triton
    (src/kernels/triton_paged_attention.py:220)."""
    return _attn_call("prefill", q, k_pool, v_pool, page_table, seq_lens, current_lengths)


def paged_attention(backend: str, q: torch.Tensor, kv_cache, current_lengths) -> torch.Tensor:
    """Attention of ``q [B,H,T,D]`` over the paged cache of ``kv_cache``.

    Same contract as src/kernels/paged_attention.py:13-51 for the GPU backend.
    ``kv_cache`` may be this package's BatchedPagedKVCache or the reference's
    (only ``states``, ``states[i].block_ids``/``seq_len`` and ``pool.k_blocks``
    / ``v_blocks`` are read).
    """
    if backend not in SUPPORTED_BACKENDS:
        raise ValueError(f"Unsupported paged attention backend: {backend}")
    if not q.is_cuda:
        raise RuntimeError("b2pa: q must be a CUDA tensor (this package has no CPU path)")
    B, _, T, _ = q.shape
    dev = q.device
    # host-side current lengths as one int32 metadata row (a scalar stands for
    # a row of equal values)
    host_cur = None
    if current_lengths is None:
        host_cur = T
    elif isinstance(current_lengths, int):
        host_cur = current_lengths
    elif isinstance(current_lengths, torch.Tensor) and not current_lengths.is_cuda:
        host_cur = current_lengths.numpy()
    elif isinstance(current_lengths, (list, tuple)):
        host_cur = [int(x) for x in current_lengths]
    pool = kv_cache.pool
    pend = getattr(pool, "_b2pa_pending", None)
    step = getattr(pool, "_b2pa_step", None)
    if step is not None:  # an open DecodeStep: its shared metadata, no host work
        if not isinstance(pend, _StepPending) or pend.step is not step or T != 1:
            raise RuntimeError("b2pa: inside a DecodeStep, paged_attention must follow its layer's append_batch")
        step.layer_of(kv_cache)
        pool._b2pa_pending = None
        return step.attend(q, kv_cache, pend)
    if pend is not None:
        if (pend.cache is kv_cache and pend.k_new.shape[2] == T and pend.k_new.device == dev
                and pool.k_blocks.dtype == q.dtype):
            if T == 1:
                return _decode_with_append(q, kv_cache, current_lengths, host_cur, take_pending(pool))
            return _prefill_with_append(q, kv_cache, current_lengths, host_cur, take_pending(pool))
        flush_pending(pool)
    if pool.k_blocks is None:
        # Nothing was ever appended to this layer: every row sees no key, which
        # the reference defines as a zero output (reference_paged_attention.py:16,51-52).
        return torch.zeros_like(q)
    if host_cur is not None:
        page_table, seq_lens, cur, max_pages = block_table_and_lengths(kv_cache, dev, [host_cur], transient=True)
    else:
        page_table, seq_lens, max_pages = block_table_and_lengths(kv_cache, dev, transient=True)
        cur = current_lengths.to(dtype=torch.int32)
    fn = "decode" if T == 1 else "prefill"
    return _attn_call(fn, q, pool.k_blocks, pool.v_blocks, page_table, seq_lens, cur, max_pages)


def _decode_with_append(q, kv_cache, current_lengths, host_cur, pend) -> torch.Tensor:
    """Decode of ``q`` with the deferred append ``pend`` of the same batch
    performed in the same launch (b2pa_paged_decode_append): the pair
    append_batch + paged_attention of src/model/attention.py:56-62."""
    pool = kv_cache.pool
    kb, vb = pool.k_blocks, pool.v_blocks
    dev = q.device
    B, H, _, D = q.shape
    if host_cur is not None:
        page_table, seq_lens, cur, start_t, len_t, max_pages = block_table_and_lengths(
            kv_cache, dev, [host_cur, pend.starts, pend.lengths], transient=True)
    else:
        page_table, seq_lens, start_t, len_t, max_pages = block_table_and_lengths(
            kv_cache, dev, [pend.starts, pend.lengths], transient=True)
        cur = current_lengths.to(dtype=torch.int32)
    out = torch.empty_like(q)
    dt = _lib.dtype_code(q.dtype)
    lib = _lib.load()
    block_size = kb.shape[2]
    ws_bytes = lib.b2pa_paged_decode_workspace_size(B, H, D, max_pages, block_size, dt)
    ws = _lib.workspace(dev, ws_bytes) if ws_bytes else None
    k_new, v_new = pend.k_new, pend.v_new
    rc = lib.b2pa_paged_decode_append(
        q.data_ptr(), _lib.strides4(q), k_new.data_ptr(), _lib.strides4(k_new), v_new.data_ptr(),
        _lib.strides4(v_new), kb.data_ptr(), vb.data_ptr(), _lib.strides4(kb), kb.shape[0],
        page_table.data_ptr() if max_pages else None, page_table.stride(0), max_pages,
        seq_lens.data_ptr(), cur.data_ptr(), start_t.data_ptr(), len_t.data_ptr(), pend.seq_out.data_ptr(),
        out.data_ptr(), _lib.strides4(out), B, H, D, block_size, 1.0 / math.sqrt(D), dt,
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        _lib.status_buffer(dev).data_ptr(), _lib.stream_handle(dev))
    if rc != 0:
        # Nothing was launched.  Append with the ordinary kernel so the pool
        # ends as the reference's append leaves it; a layout the fused entry
        # does not take (rows not 4-byte aligned) then decodes separately.
        err = _lib.last_error()
        seq = _kv_append(kv_cache, k_new, v_new, pend.starts, pend.lengths)
        pend.seq_out.copy_(seq)
        if rc == _lib.STATUS_CODES["B2PA_ERR_UNSUPPORTED"]:
            return _attn_call("decode", q, kb, vb, page_table, seq_lens, cur, max_pages)
        raise RuntimeError(f"b2pa_paged_decode_append failed: {_lib.STATUS_NAMES.get(rc, rc)}: {err}")
    return out


def _prefill_with_append(q, kv_cache, current_lengths, host_cur, pend) -> torch.Tensor:
    """Chunked prefill of ``q`` with the deferred append ``pend`` of the same
    batch (b2pa_paged_prefill_append): for fp32 pools with head_dim 64 the
    append happens inside the page copy of the tensor-core path, otherwise
    the append kernel runs first."""
    pool = kv_cache.pool
    kb, vb = pool.k_blocks, pool.v_blocks
    dev = q.device
    B, H, T, D = q.shape
    if host_cur is not None:
        page_table, seq_lens, cur, start_t, len_t, max_pages = block_table_and_lengths(
            kv_cache, dev, [host_cur, pend.starts, pend.lengths], transient=True)
    else:
        page_table, seq_lens, start_t, len_t, max_pages = block_table_and_lengths(
            kv_cache, dev, [pend.starts, pend.lengths], transient=True)
        cur = current_lengths.to(dtype=torch.int32)
    out = torch.empty_like(q)
    dt = _lib.dtype_code(q.dtype)
    lib = _lib.load()
    block_size = kb.shape[2]
    ws_bytes = lib.b2pa_paged_prefill_workspace_size(B, H, T, D, max_pages, block_size, dt)
    ws = _lib.workspace(dev, ws_bytes) if ws_bytes else None
    k_new, v_new = pend.k_new, pend.v_new
    rc = lib.b2pa_paged_prefill_append(
        q.data_ptr(), _lib.strides4(q), k_new.data_ptr(), _lib.strides4(k_new), v_new.data_ptr(),
        _lib.strides4(v_new), kb.data_ptr(), vb.data_ptr(), _lib.strides4(kb), kb.shape[0],
        page_table.data_ptr() if max_pages else None, page_table.stride(0), max_pages,
        seq_lens.data_ptr(), cur.data_ptr(), start_t.data_ptr(), len_t.data_ptr(), pend.seq_out.data_ptr(),
        out.data_ptr(), _lib.strides4(out), B, H, T, D, block_size, 1.0 / math.sqrt(D), dt,
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        _lib.status_buffer(dev).data_ptr(), _lib.stream_handle(dev))
    if rc != 0:
        # The attention did not run.  On the non-fused path the append kernel
        # may already have been queued; appending again with the ordinary
        # kernel writes the same bytes, and leaves the pool as the
        # reference's append does either way.  Then report.
        err = _lib.last_error()
        seq = _kv_append(kv_cache, k_new, v_new, pend.starts, pend.lengths)
        pend.seq_out.copy_(seq)
        raise RuntimeError(f"b2pa_paged_prefill_append failed: {_lib.STATUS_NAMES.get(rc, rc)}: {err}")
    return out
