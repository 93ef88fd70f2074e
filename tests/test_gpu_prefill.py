"""Chunked-prefill paged attention on the GPU against the reference's golden
outputs and the CPU oracle (fp32: rtol 1e-4 / atol 1e-5; bf16/fp16: 2e-2)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import b2pa
from oracle import oracle as orc
from tests._helpers import TOL, build_cache, golden_tensor, load_golden, random_tables, split_tables, strided_q

pytestmark = pytest.mark.gpu


def _check(out: torch.Tensor, ref: np.ndarray, dtype) -> None:
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, **TOL[dtype])


@pytest.mark.parametrize("name", ["prefill_f32_bs16_d32", "prefill_f32_bs8_d16", "prefill_bf16_bs16_d64"])
def test_golden_prefill(cuda_device, name):
    g = load_golden(name)
    dt = str(g["dtype"])
    dtype = torch.bfloat16 if dt == "bfloat16" else torch.float32
    kp = golden_tensor(g["k_pool"], dt).to(cuda_device)
    vp = golden_tensor(g["v_pool"], dt).to(cuda_device)
    q = golden_tensor(g["q"], dt).to(cuda_device)
    tables = split_tables(g["block_ids"], g["block_counts"])
    cache = build_cache(b2pa, kp, vp, tables, g["seq_lens"].tolist(), int(g["block_size"]))
    out = b2pa.paged_attention("b200_paged", q, cache, torch.tensor(g["cur_lens"]))
    _check(out, g["out"], dtype)
    assert b2pa.read_status(cuda_device) == 0


def _random_prefill(device, *, B, H, D, bs, T, dtype, prefixes, curs, seed):
    rng = np.random.default_rng(seed)
    gen = torch.Generator().manual_seed(seed)
    lens = [p + c for p, c in zip(prefixes, curs)]
    NB = sum(-(-L // bs) for L in lens) + 5
    kp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    vp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    tables = random_tables(rng, lens, NB, bs)
    cache = build_cache(b2pa, kp, vp, tables, lens, bs)
    q = strided_q(B, H, T, D, dtype, device, gen)
    out = b2pa.paged_attention("b200_paged", q, cache, torch.tensor(curs))
    ref = orc.paged_attention_c(q.float().cpu().numpy(), kp.float().cpu().numpy(), vp.float().cpu().numpy(), tables,
                                lens, curs)
    assert out.stride() == q.stride()  # empty_like(q), as the reference launchers
    return out, ref


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_config2_prefill(cuda_device, dtype):
    """B=8, 256-token chunk over a cached prefix
    P ~ U[0,768], H=8, D=64, block 16."""
    rng = np.random.default_rng(2)
    prefixes = rng.integers(0, 769, size=8).tolist()
    out, ref = _random_prefill(cuda_device, B=8, H=8, D=64, bs=16, T=256, dtype=dtype, prefixes=prefixes,
                               curs=[256] * 8, seed=2)
    _check(out, ref, dtype)
    assert b2pa.read_status(cuda_device) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D,bs", [(16, 8), (32, 16), (64, 16), (128, 16), (256, 32), (64, 32), (128, 8)])
def test_prefill_shapes_with_padding(cuda_device, dtype, D, bs):
    # padded rows (cur < T), a zero-length row, T not a multiple of 32
    T = 45
    out, ref = _random_prefill(cuda_device, B=4, H=3, D=D, bs=bs, T=T, dtype=dtype, prefixes=[0, 13, 70, 5],
                               curs=[45, 20, 0, 1], seed=D * 3 + bs)
    _check(out, ref, dtype)


def test_prefill_first_chunk_and_continuation(cuda_device):
    # chunked prefill as the continuous scheduler runs it: same chunk start
    out, ref = _random_prefill(cuda_device, B=5, H=8, D=64, bs=16, T=128, dtype=torch.float32,
                               prefixes=[256, 256, 256, 256, 256], curs=[128, 128, 60, 1, 128], seed=3)
    _check(out, ref, torch.float32)


def test_prefill_through_append(cuda_device):
    """append_batch then paged_attention, as CausalSelfAttention.forward does
    (src/model/attention.py:56-62), checked against the oracle's append."""
    torch.manual_seed(7)
    B, H, D, bs = 3, 4, 64, 16
    pool = b2pa.LayerBlockPool(bs, 4, 2.0)
    cache = b2pa.BatchedPagedKVCache([b2pa.PagedKVCacheState(pool=pool) for _ in range(B)], pool=pool)
    mpool = orc.OraclePool(bs, 4, 2.0)
    mstates = [orc.OracleState(mpool) for _ in range(B)]
    for T, lens in [(50, [50, 31, 7]), (64, [64, 64, 64]), (1, [1, 1, 1]), (20, [3, 20, 0])]:
        x = torch.randn(B, T, 3, H, D)
        k, v, q = (x[:, :, i].transpose(1, 2) for i in range(3))
        cache.append_batch(k.cuda(), v.cuda(), torch.tensor(lens))
        orc.oracle_append_batch(mstates, k.numpy(), v.numpy(), lens)
        out = b2pa.paged_attention("b200_paged", q.cuda(), cache, torch.tensor(lens, device="cuda"))
        ref = orc.paged_attention_c(q.numpy(), mpool.k, mpool.v, [s.block_ids for s in mstates],
                                    [s.seq_len for s in mstates], lens)
        _check(out, ref, torch.float32)
    assert b2pa.read_status(cuda_device) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
def test_prefill_tensor_core_multi_tile(cuda_device, dtype, D):
    # several 128-row query tiles, long prefixes, chunk rows padded at the end
    out, ref = _random_prefill(cuda_device, B=3, H=2, D=D, bs=16, T=300, dtype=dtype, prefixes=[0, 500, 1000],
                               curs=[300, 171, 300], seed=D)
    _check(out, ref, dtype)
    assert b2pa.read_status(cuda_device) == 0


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_prefill_f32_multi_tile(cuda_device, D, bs):
    # fp32 kernels -- head_dim 64: tensor cores on fp16 hi/lo splits (here
    # with a key-range split and its combine); 128: register-tiled CUDA cores
    # -- several query and key tiles, a short and an empty sequence, rows
    # padded past cur_len
    out, ref = _random_prefill(cuda_device, B=4, H=3, D=D, bs=bs, T=200, dtype=torch.float32,
                               prefixes=[0, 333, 1000, 0], curs=[200, 97, 200, 0], seed=D + bs)
    _check(out, ref, torch.float32)
    assert b2pa.read_status(cuda_device) == 0


def test_prefill_f32_bad_block_id_is_reported(cuda_device):
    torch.manual_seed(2)
    kp = torch.randn(4, 2, 16, 64, device=cuda_device)
    vp = torch.randn_like(kp)
    cache = build_cache(b2pa, kp, vp, [[0, 9, 1]], [40], 16)  # block 9 is past the pool
    b2pa.clear_status(cuda_device)
    q = torch.randn(1, 2, 20, 64, device=cuda_device)
    out = b2pa.paged_attention("b200_paged", q, cache, 20)
    assert b2pa.read_status(cuda_device) == -3
    b2pa.clear_status(cuda_device)
    assert torch.isfinite(out).all()


def test_prefill_bad_block_id_is_reported(cuda_device):
    torch.manual_seed(1)
    kp = torch.randn(4, 2, 16, 64, device=cuda_device, dtype=torch.bfloat16)
    vp = torch.randn_like(kp)
    cache = build_cache(b2pa, kp, vp, [[0, 9, 1]], [40], 16)  # block 9 is past the pool
    b2pa.clear_status(cuda_device)
    q = torch.randn(1, 2, 20, 64, device=cuda_device, dtype=torch.bfloat16)
    out = b2pa.paged_attention("b200_paged", q, cache, 20)
    assert b2pa.read_status(cuda_device) == -3
    b2pa.clear_status(cuda_device)
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("D", [64, 128])
def test_prefill_tensor_core_key_split(cuda_device, D):
    # few (query tile, head, sequence) CTAs: the key range is split across
    # CTAs and merged by the combine kernel; the second sequence is short, so
    # its tiles need fewer splits than the first's
    out, ref = _random_prefill(cuda_device, B=2, H=3, D=D, bs=16, T=200, dtype=torch.bfloat16,
                               prefixes=[1500, 20], curs=[200, 130], seed=5 + D)
    _check(out, ref, torch.bfloat16)
    assert b2pa.read_status(cuda_device) == 0


@pytest.mark.parametrize("where", ["k", "v", "q"])
def test_prefill_f32_outside_split_range_is_recomputed(cuda_device, where):
    """fp32 head_dim 64 runs on the tensor cores with fp16 hi/lo splits of its
    operands, which hold |x| < 2^15 only; an input at or beyond that (in K, V
    or q) sends the call to the fp32 CUDA-core kernel, so the result still
    matches the oracle."""
    rng = np.random.default_rng(17)
    gen = torch.Generator().manual_seed(17)
    B, H, D, bs, T = 3, 2, 64, 16, 40
    prefixes, curs = [30, 0, 90], [40, 25, 40]
    lens = [p + c for p, c in zip(prefixes, curs)]
    NB = sum(-(-L // bs) for L in lens) + 2
    kp = torch.randn(NB, H, bs, D, generator=gen) * 0.01
    vp = torch.randn(NB, H, bs, D, generator=gen)
    tables = random_tables(rng, lens, NB, bs)
    q = strided_q(B, H, T, D, torch.float32, "cpu", gen) * 0.01
    big = 4.0e4
    if where == "k":
        kp[tables[2][1], 1, 3, 5] = big  # one key entry of a visible page
    elif where == "v":
        vp[tables[0][0], 0, 7, 60] = -big
    else:
        q[1, 0, 2, 11] = big
    kp, vp, q = kp.to(cuda_device), vp.to(cuda_device), q.to(cuda_device)
    cache = build_cache(b2pa, kp, vp, tables, lens, bs)
    out = b2pa.paged_attention("b200_paged", q, cache, torch.tensor(curs))
    ref = orc.paged_attention_c(q.cpu().numpy(), kp.cpu().numpy(), vp.cpu().numpy(), tables, lens, curs)
    _check(out, ref, torch.float32)
    assert np.isfinite(out.cpu().numpy()).all()
    assert b2pa.read_status(cuda_device) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill_q_layout_without_tensor_map(cuda_device, dtype):
    """16-bit q is loaded with a TMA tensor map when its layout allows one;
    a q expanded along the batch (stride 0) is refused by the map encoder,
    and the kernel then loads Q with its softmax threads -- same results."""
    rng = np.random.default_rng(41)
    gen = torch.Generator().manual_seed(41)
    B, H, D, bs, T = 3, 2, 64, 16, 150
    prefixes, curs = [40, 0, 300], [150, 90, 150]
    lens = [p + c for p, c in zip(prefixes, curs)]
    NB = sum(-(-L // bs) for L in lens) + 4
    kp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(cuda_device)
    vp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(cuda_device)
    tables = random_tables(rng, lens, NB, bs)
    cache = build_cache(b2pa, kp, vp, tables, lens, bs)
    q1 = torch.randn(1, H, T, D, generator=gen).to(dtype).to(cuda_device)
    q = q1.expand(B, H, T, D)
    assert q.stride(0) == 0
    out = b2pa.paged_attention("b200_paged", q, cache, torch.tensor(curs))
    ref = orc.paged_attention_c(q.float().cpu().numpy(), kp.float().cpu().numpy(), vp.float().cpu().numpy(), tables,
                                lens, curs)
    _check(out, ref, dtype)
    assert b2pa.read_status(cuda_device) == 0
