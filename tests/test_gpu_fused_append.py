"""Decode with the KV append fused into its launch (b2pa_paged_decode_append)
and the deferred append_batch that feeds it.

* C ABI: the fused call leaves pools bit-identical to b2pa_kv_append followed
  by b2pa_paged_decode, and its output is bit-identical to that pair's (same
  bytes, same arithmetic); the output also matches the CPU oracle (fp32
  rtol 1e-4 / atol 1e-5; bf16/fp16 2e-2).  Cases: every dtype, head dims
  16-256, block sizes 8/16/32, head groupings, empty sequences growing to one
  token, appends at the first / last row of a block, rows without an append,
  cur_len 0/1/2/large (a cur_len of 2 hides the new token), split sequences.
* Bad inputs are reported through the status word without touching memory
  outside the pool.
* Chunked prefill with its append (b2pa_paged_prefill_append): pools and
  outputs bit-identical to b2pa_kv_append + b2pa_paged_prefill, on the fp32
  tensor-core path (append inside the page copy) and the others.
* Python: with ``b2pa.set_fused_append(True)`` a prefill + decode loop through
  ``append_batch`` + ``paged_attention`` (the reference's order,
  src/model/attention.py:56-62) gives the same outputs, returned lengths and
  pools as the eager path, including pool growth, a release between the two
  calls and two appends in a row.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import b2pa
from b2pa import _lib
from oracle import oracle as orc
from tests._helpers import TOL, random_tables

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    return t.view(torch.int32).numpy() if t.element_size() == 4 else t.view(torch.int16).numpy()


def _i32(vals, device):
    return torch.tensor(list(vals), dtype=torch.int32, device=device)


def _problem(device, *, H, D, bs, dtype, lens_old, cur, app=None, seed=0):
    """Pools, table and new rows for one decode step whose appends take
    lens_old[b] -> lens_old[b] + app[b]; app defaults to the reference's
    clamp(cur, 0, 1) (src/cache/paged_kv.py:167)."""
    rng = np.random.default_rng(seed)
    gen = torch.Generator().manual_seed(seed)
    B = len(lens_old)
    app = [max(min(c, 1), 0) for c in cur] if app is None else app
    lens_new = [L + a for L, a in zip(lens_old, app)]
    pages = sum(-(-L // bs) for L in lens_new)
    NB = pages + 5
    kp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    vp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    tables = random_tables(rng, lens_new, NB, bs)
    width = max(max(len(t) for t in tables), 1) + 2
    table = np.full((B, width), -1, dtype=np.int32)
    for b, t in enumerate(tables):
        table[b, :len(t)] = t
    # q, k_new, v_new as the model makes them: [B,H,1,D] views of one projection
    x = torch.randn(B, 1, 3, H, D, generator=gen).to(dtype).to(device)
    q, k_new, v_new = (x[:, :, i].transpose(1, 2) for i in range(3))
    return dict(B=B, H=H, D=D, bs=bs, dtype=dtype, kp=kp, vp=vp, tables=tables,
                table=torch.from_numpy(table).to(device), width=width, max_pages=width, q=q, k_new=k_new,
                v_new=v_new, lens_old=lens_old, lens_new=lens_new, app=app, cur=cur, NB=NB)


def _workspace(pr, device):
    lib = _lib.load()
    n = lib.b2pa_paged_decode_workspace_size(pr["B"], pr["H"], pr["D"], pr["max_pages"], pr["bs"],
                                             _lib.dtype_code(pr["dtype"]))
    return torch.empty(max(n, 1) + 256, dtype=torch.uint8, device=device)


def _unfused(pr, device):
    lib = _lib.load()
    kp, vp = pr["kp"].clone(), pr["vp"].clone()
    st = _lib.status_buffer(device).data_ptr()
    sh = _lib.stream_handle(device)
    dt = _lib.dtype_code(pr["dtype"])
    starts, lens, seq, cur = (_i32(pr["lens_old"], device), _i32(pr["app"], device), _i32(pr["lens_new"], device),
                              _i32(pr["cur"], device))
    _lib.check(lib.b2pa_kv_append(pr["k_new"].data_ptr(), _lib.strides4(pr["k_new"]), pr["v_new"].data_ptr(),
                                  _lib.strides4(pr["v_new"]), kp.data_ptr(), vp.data_ptr(), _lib.strides4(kp),
                                  pr["NB"], pr["table"].data_ptr(), pr["width"], pr["max_pages"], starts.data_ptr(),
                                  lens.data_ptr(), pr["B"], pr["H"], 1, pr["D"], pr["bs"], dt, st, sh), "append")
    out = torch.empty_like(pr["q"])
    ws = _workspace(pr, device)
    _lib.check(lib.b2pa_paged_decode(pr["q"].data_ptr(), _lib.strides4(pr["q"]), kp.data_ptr(), vp.data_ptr(),
                                     _lib.strides4(kp), pr["NB"], pr["table"].data_ptr(), pr["width"],
                                     pr["max_pages"], seq.data_ptr(), cur.data_ptr(), out.data_ptr(),
                                     _lib.strides4(out), pr["B"], pr["H"], pr["D"], pr["bs"],
                                     1.0 / math.sqrt(pr["D"]), dt, ws.data_ptr(), ws.numel(), st, sh), "decode")
    torch.cuda.synchronize()
    return out, kp, vp


def _fused(pr, device, starts=None):
    lib = _lib.load()
    kp, vp = pr["kp"].clone(), pr["vp"].clone()
    starts = _i32(pr["lens_old"] if starts is None else starts, device)
    lens, seq, cur = _i32(pr["app"], device), _i32(pr["lens_new"], device), _i32(pr["cur"], device)
    seq_out = torch.full((pr["B"],), -7, dtype=torch.int64, device=device)
    out = torch.empty_like(pr["q"])
    ws = _workspace(pr, device)
    rc = lib.b2pa_paged_decode_append(
        pr["q"].data_ptr(), _lib.strides4(pr["q"]), pr["k_new"].data_ptr(), _lib.strides4(pr["k_new"]),
        pr["v_new"].data_ptr(), _lib.strides4(pr["v_new"]), kp.data_ptr(), vp.data_ptr(), _lib.strides4(kp),
        pr["NB"], pr["table"].data_ptr(), pr["width"], pr["max_pages"], seq.data_ptr(), cur.data_ptr(),
        starts.data_ptr(), lens.data_ptr(), seq_out.data_ptr(), out.data_ptr(), _lib.strides4(out), pr["B"],
        pr["H"], pr["D"], pr["bs"], 1.0 / math.sqrt(pr["D"]), _lib.dtype_code(pr["dtype"]), ws.data_ptr(),
        ws.numel(), _lib.status_buffer(device).data_ptr(), _lib.stream_handle(device))
    _lib.check(rc, "b2pa_paged_decode_append")
    torch.cuda.synchronize()
    return out, kp, vp, seq_out


def _compare(pr, device):
    b2pa.clear_status(device)
    out_a, kp_a, vp_a = _unfused(pr, device)
    assert b2pa.read_status(device) == 0
    out_b, kp_b, vp_b, seq_out = _fused(pr, device)
    assert b2pa.read_status(device) == 0
    assert np.array_equal(_bits(kp_a), _bits(kp_b))
    assert np.array_equal(_bits(vp_a), _bits(vp_b))
    assert np.array_equal(_bits(out_a), _bits(out_b))
    assert seq_out.tolist() == pr["lens_new"]
    ref = orc.paged_attention_c(pr["q"].float().cpu().numpy(), kp_b.float().cpu().numpy(),
                                vp_b.float().cpu().numpy(), pr["tables"], pr["lens_new"], pr["cur"])
    np.testing.assert_allclose(out_b.float().cpu().numpy(), ref, **TOL[pr["dtype"]])


# lengths before the step: empty, a block's last row / first row next, split sequences
_LENS = [0, 15, 16, 31, 32, 100, 299, 7, 650]
_CUR = [1, 1, 1, 1, 1, 1, 1, 0, 1]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D,bs", [(64, 16), (128, 16), (16, 8), (256, 32), (32, 8)])
def test_fused_equals_append_then_decode(cuda_device, dtype, D, bs):
    pr = _problem(cuda_device, H=4, D=D, bs=bs, dtype=dtype, lens_old=_LENS, cur=_CUR, seed=D + bs)
    _compare(pr, cuda_device)


@pytest.mark.parametrize("H", [1, 3, 6, 12])
def test_fused_head_groupings(cuda_device, H):
    pr = _problem(cuda_device, H=H, D=64, bs=16, dtype=torch.float32, lens_old=_LENS, cur=_CUR, seed=H)
    _compare(pr, cuda_device)


def test_fused_current_lengths(cuda_device):
    # cur 2: the new token is appended but not visible; cur 30 > length: no key
    # visible, zero output; app given apart from cur (the ABI allows it)
    lens_old = [40, 40, 16, 0, 3, 200]
    cur = [2, 30, 0, 1, 5, 1]
    app = [1, 1, 1, 1, 0, 1]
    pr = _problem(cuda_device, H=4, D=64, bs=16, dtype=torch.float32, lens_old=lens_old, cur=cur, app=app, seed=5)
    _compare(pr, cuda_device)


def test_fused_long_sequences_bf16(cuda_device):
    # config[4]-like rows (H=32, D=128, bf16): many splits per sequence
    rng = np.random.default_rng(3)
    lens_old = rng.integers(1024, 4096, size=6).tolist()
    pr = _problem(cuda_device, H=32, D=128, bs=16, dtype=torch.bfloat16, lens_old=lens_old, cur=[1] * 6, seed=3)
    _compare(pr, cuda_device)


def test_fused_contiguous_split(cuda_device):
    # 1200 sequences x 2 head groups: the contiguous split, with the append
    # done by the CTA whose piece holds each stream's last page
    rng = np.random.default_rng(12)
    lens_old = rng.integers(0, 150, size=1200)
    lens_old[:4] = [0, 15, 16, 31]
    lens_old[500], lens_old[1199] = 7000, 4097
    cur = [1] * 1200
    cur[4], cur[5] = 2, 0
    pr = _problem(cuda_device, H=8, D=16, bs=16, dtype=torch.bfloat16, lens_old=lens_old.tolist(), cur=cur, seed=12)
    _compare(pr, cuda_device)


def test_fused_bad_position_and_block_reported(cuda_device):
    """A start position other than seq_len - 1 and a block id past the pool
    end are skipped and reported; the pools keep their bytes."""
    pr = _problem(cuda_device, H=2, D=64, bs=16, dtype=torch.float32, lens_old=[20, 20], cur=[1, 1], seed=9)
    b2pa.clear_status(cuda_device)
    _, kp, vp, _ = _fused(pr, cuda_device, starts=[20, 5])  # row 1 claims position 5
    assert b2pa.read_status(cuda_device) == _lib.STATUS_CODES["B2PA_ERR_INVALID_ARGUMENT"]
    b2pa.clear_status(cuda_device)
    for blk in pr["tables"][1]:  # neither the claimed nor the real position was written
        assert torch.equal(kp[blk], pr["kp"][blk]) and torch.equal(vp[blk], pr["vp"][blk])
    new_blk = pr["tables"][0][1]
    assert torch.equal(kp[new_blk, :, 4], pr["k_new"][0, :, 0])  # row 0 (valid) landed
    pr["table"][0, 1] = pr["NB"] + 3  # the page of row 0's new token
    _, kp, vp, _ = _fused(pr, cuda_device)
    assert b2pa.read_status(cuda_device) == _lib.STATUS_CODES["B2PA_ERR_BAD_BLOCK_ID"]
    b2pa.clear_status(cuda_device)
    for blk in pr["tables"][0]:  # row 0's append was skipped
        assert torch.equal(kp[blk], pr["kp"][blk]) and torch.equal(vp[blk], pr["vp"][blk])
    assert torch.equal(kp[pr["tables"][1][1], :, 4], pr["k_new"][1, :, 0])  # row 1's append landed


# ------------------------------------------------------------ Python layer
def _decode_loop(device, dtype, fused: bool):
    """Prefill + decode steps through append_batch / paged_attention; returns
    outputs, returned lengths and the final pools."""
    prev = b2pa.set_fused_append(fused)
    try:
        gen = torch.Generator().manual_seed(11)
        B, H, D, bs = 5, 4, 64, 16
        pool = b2pa.LayerBlockPool(bs, 3, 2.0)  # small: the decode steps grow it
        states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(B)]
        outs, rets = [], []

        def rows(T):
            x = torch.randn(B, T, 3, H, D, generator=gen).to(dtype).to(device)
            return (x[:, :, i].transpose(1, 2) for i in range(3))

        cache = b2pa.BatchedPagedKVCache(states, pool=pool)
        q, k, v = rows(20)
        rets.append(cache.append_batch(k, v, torch.tensor([20, 3, 17, 0, 9])))
        outs.append(b2pa.paged_attention("b200_paged", q, cache, torch.tensor([20, 3, 17, 0, 9])))
        for step in range(40):
            cache = b2pa.BatchedPagedKVCache(states, pool=pool)  # a new batch object per step, as the reference
            q, k, v = rows(1)
            cur = 1 if step % 3 else torch.tensor([1, 1, 0, 1, 2])
            rets.append(cache.append_batch(k, v, cur))
            if step == 17:
                states[3].release()  # between the append and the attention
            if step == 25:  # two appends in a row: the first one must land
                q2, k2, v2 = rows(1)
                rets.append(cache.append_batch(k2, v2, 1))
            outs.append(b2pa.paged_attention("b200_paged", q, cache, cur))
        torch.cuda.synchronize()
        assert getattr(pool, "_b2pa_pending", None) is None
        return outs, [r.tolist() for r in rets], pool.k_blocks.clone(), pool.v_blocks.clone(), \
            [list(s.block_ids) for s in states]
    finally:
        b2pa.set_fused_append(prev)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_deferred_append_matches_eager(cuda_device, dtype):
    b2pa.clear_status(cuda_device)
    outs_e, rets_e, kp_e, vp_e, ids_e = _decode_loop(cuda_device, dtype, fused=False)
    outs_f, rets_f, kp_f, vp_f, ids_f = _decode_loop(cuda_device, dtype, fused=True)
    assert b2pa.read_status(cuda_device) == 0
    assert ids_e == ids_f
    assert rets_e == rets_f
    assert np.array_equal(_bits(kp_e), _bits(kp_f))
    assert np.array_equal(_bits(vp_e), _bits(vp_f))
    for a, b in zip(outs_e, outs_f):
        assert np.array_equal(_bits(a), _bits(b))


def test_flush_pending_writes_the_row(cuda_device):
    prev = b2pa.set_fused_append(True)
    try:
        pool = b2pa.LayerBlockPool(16, 4, 2.0)
        states = [b2pa.PagedKVCacheState(pool=pool) for _ in range(2)]
        cache = b2pa.BatchedPagedKVCache(states, pool=pool)
        k = torch.randn(2, 3, 1, 32, device=cuda_device)
        v = torch.randn(2, 3, 1, 32, device=cuda_device)
        ret = cache.append_batch(k, v, 1)
        assert pool._b2pa_pending is not None
        b2pa.flush_pending(pool)
        assert pool._b2pa_pending is None
        assert ret.tolist() == [1, 1]
        for b, s in enumerate(states):
            assert torch.equal(pool.k_blocks[s.block_ids[0], :, 0], k[b, :, 0])
            assert torch.equal(pool.v_blocks[s.block_ids[0], :, 0], v[b, :, 0])
    finally:
        b2pa.set_fused_append(prev)


# ---------------------------------------------- chunked prefill with its append
def _prefill_problem(device, *, H, D, bs, T, dtype, prefixes, app, seed):
    """Pools and table for one prompt chunk per sequence: app[b] <= T new
    tokens after prefixes[b] cached ones."""
    rng = np.random.default_rng(seed)
    gen = torch.Generator().manual_seed(seed)
    B = len(prefixes)
    lens_new = [p + a for p, a in zip(prefixes, app)]
    NB = sum(-(-L // bs) for L in lens_new) + 4
    kp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    vp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    tables = random_tables(rng, lens_new, NB, bs)
    width = max(max(len(t) for t in tables), 1) + 1
    table = np.full((B, width), -1, dtype=np.int32)
    for b, t in enumerate(tables):
        table[b, :len(t)] = t
    x = torch.randn(B, T, 3, H, D, generator=gen).to(dtype).to(device)
    q, k_new, v_new = (x[:, :, i].transpose(1, 2) for i in range(3))
    return dict(B=B, H=H, D=D, bs=bs, T=T, dtype=dtype, kp=kp, vp=vp, tables=tables,
                table=torch.from_numpy(table).to(device), width=width, q=q, k_new=k_new, v_new=v_new,
                starts=list(prefixes), app=list(app), lens_new=lens_new, NB=NB)


def _prefill_ws(pr, device):
    n = _lib.load().b2pa_paged_prefill_workspace_size(pr["B"], pr["H"], pr["T"], pr["D"], pr["width"], pr["bs"],
                                                      _lib.dtype_code(pr["dtype"]))
    return torch.empty(max(n, 1) + 256, dtype=torch.uint8, device=device)


def _prefill_unfused(pr, device):
    lib = _lib.load()
    kp, vp = pr["kp"].clone(), pr["vp"].clone()
    st, sh, dt = _lib.status_buffer(device).data_ptr(), _lib.stream_handle(device), _lib.dtype_code(pr["dtype"])
    starts, lens, seq = _i32(pr["starts"], device), _i32(pr["app"], device), _i32(pr["lens_new"], device)
    _lib.check(lib.b2pa_kv_append(pr["k_new"].data_ptr(), _lib.strides4(pr["k_new"]), pr["v_new"].data_ptr(),
                                  _lib.strides4(pr["v_new"]), kp.data_ptr(), vp.data_ptr(), _lib.strides4(kp),
                                  pr["NB"], pr["table"].data_ptr(), pr["width"], pr["width"], starts.data_ptr(),
                                  lens.data_ptr(), pr["B"], pr["H"], pr["T"], pr["D"], pr["bs"], dt, st, sh),
               "append")
    out = torch.empty_like(pr["q"])
    ws = _prefill_ws(pr, device)
    _lib.check(lib.b2pa_paged_prefill(pr["q"].data_ptr(), _lib.strides4(pr["q"]), kp.data_ptr(), vp.data_ptr(),
                                      _lib.strides4(kp), pr["NB"], pr["table"].data_ptr(), pr["width"], pr["width"],
                                      seq.data_ptr(), lens.data_ptr(), out.data_ptr(), _lib.strides4(out), pr["B"],
                                      pr["H"], pr["T"], pr["D"], pr["bs"], 1.0 / math.sqrt(pr["D"]), dt,
                                      ws.data_ptr(), ws.numel(), st, sh), "prefill")
    torch.cuda.synchronize()
    return out, kp, vp


def _prefill_fused(pr, device, starts=None):
    lib = _lib.load()
    kp, vp = pr["kp"].clone(), pr["vp"].clone()
    starts = _i32(pr["starts"] if starts is None else starts, device)
    lens, seq = _i32(pr["app"], device), _i32(pr["lens_new"], device)
    seq_out = torch.full((pr["B"],), -7, dtype=torch.int64, device=device)
    out = torch.empty_like(pr["q"])
    ws = _prefill_ws(pr, device)
    rc = lib.b2pa_paged_prefill_append(
        pr["q"].data_ptr(), _lib.strides4(pr["q"]), pr["k_new"].data_ptr(), _lib.strides4(pr["k_new"]),
        pr["v_new"].data_ptr(), _lib.strides4(pr["v_new"]), kp.data_ptr(), vp.data_ptr(), _lib.strides4(kp),
        pr["NB"], pr["table"].data_ptr(), pr["width"], pr["width"], seq.data_ptr(), lens.data_ptr(),
        starts.data_ptr(), lens.data_ptr(), seq_out.data_ptr(), out.data_ptr(), _lib.strides4(out), pr["B"],
        pr["H"], pr["T"], pr["D"], pr["bs"], 1.0 / math.sqrt(pr["D"]), _lib.dtype_code(pr["dtype"]),
        ws.data_ptr(), ws.numel(), _lib.status_buffer(device).data_ptr(), _lib.stream_handle(device))
    _lib.check(rc, "b2pa_paged_prefill_append")
    torch.cuda.synchronize()
    return out, kp, vp, seq_out


@pytest.mark.parametrize("dtype,D,bs", [(torch.float32, 64, 16), (torch.float32, 64, 8), (torch.float32, 64, 32),
                                        (torch.float32, 128, 16), (torch.bfloat16, 64, 16),
                                        (torch.float16, 128, 32)])
def test_prefill_append_equals_append_then_prefill(cuda_device, dtype, D, bs):
    """b2pa_paged_prefill_append (fp32 head_dim 64: the append inside the
    tensor-core path's page copy; otherwise append kernel + prefill) leaves
    the same pool bytes and output as b2pa_kv_append + b2pa_paged_prefill:
    prefixes across page boundaries, a padded chunk, an empty sequence
    growing, a sequence without new tokens."""
    pr = _prefill_problem(cuda_device, H=3, D=D, bs=bs, T=40, dtype=dtype, prefixes=[0, 13, 70, 16, 5],
                          app=[40, 25, 40, 1, 0], seed=D + bs)
    b2pa.clear_status(cuda_device)
    out_a, kp_a, vp_a = _prefill_unfused(pr, cuda_device)
    out_b, kp_b, vp_b, seq_out = _prefill_fused(pr, cuda_device)
    assert b2pa.read_status(cuda_device) == 0
    assert np.array_equal(_bits(kp_a), _bits(kp_b))
    assert np.array_equal(_bits(vp_a), _bits(vp_b))
    assert np.array_equal(_bits(out_a), _bits(out_b))
    assert seq_out.tolist() == pr["lens_new"]
    ref = orc.paged_attention_c(pr["q"].float().cpu().numpy(), kp_b.float().cpu().numpy(),
                                vp_b.float().cpu().numpy(), pr["tables"], pr["lens_new"], pr["app"])
    np.testing.assert_allclose(out_b.float().cpu().numpy(), ref, **TOL[dtype])


def test_prefill_append_refuses_a_chunk_that_does_not_end_the_sequence(cuda_device):
    pr = _prefill_problem(cuda_device, H=2, D=64, bs=16, T=20, dtype=torch.float32, prefixes=[30, 10],
                          app=[20, 20], seed=4)
    b2pa.clear_status(cuda_device)
    _, kp, vp, _ = _prefill_fused(pr, cuda_device, starts=[30, 3])  # row 1 claims positions 3..22
    assert b2pa.read_status(cuda_device) == _lib.STATUS_CODES["B2PA_ERR_INVALID_ARGUMENT"]
    b2pa.clear_status(cuda_device)
    for blk in pr["tables"][1]:  # sequence 1 was not written
        assert torch.equal(kp[blk], pr["kp"][blk]) and torch.equal(vp[blk], pr["vp"][blk])
    assert torch.equal(kp[pr["tables"][0][2], :, 0], pr["k_new"][0, :, 2])  # position 32 of sequence 0 was
