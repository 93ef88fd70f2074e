"""Paged decode attention on the GPU against the reference's golden outputs
and the CPU oracle (fp32: rtol 1e-4 / atol 1e-5; bf16/fp16: 2e-2)."""
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


@pytest.mark.parametrize("name", ["decode_f32_bs8_d16", "decode_f32_curvar", "decode_f32_bs16_d64",
                                  "decode_bf16_bs16_d128"])
def test_golden_decode(cuda_device, name):
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


def _random_decode(device, *, B, H, D, bs, dtype, lmin, lmax, seed, cur=None, nb_extra=7, lens=None):
    rng = np.random.default_rng(seed)
    gen = torch.Generator().manual_seed(seed)
    if lens is None:
        lens = rng.integers(lmin, lmax + 1, size=B).tolist()
    pages = sum(-(-L // bs) for L in lens)
    NB = pages + nb_extra
    kp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    vp = torch.randn(NB, H, bs, D, generator=gen).to(dtype).to(device)
    tables = random_tables(rng, lens, NB, bs)
    cache = build_cache(b2pa, kp, vp, tables, lens, bs)
    q = strided_q(B, H, 1, D, dtype, device, gen)
    cur = [1] * B if cur is None else cur
    out = b2pa.paged_attention("b200_paged", q, cache, torch.tensor(cur))
    ref = orc.paged_attention_c(q.float().cpu().numpy(), kp.float().cpu().numpy(), vp.float().cpu().numpy(), tables,
                                lens, cur)
    return out, ref


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_decode_shapes(cuda_device, dtype, D, bs):
    out, ref = _random_decode(cuda_device, B=5, H=4, D=D, bs=bs, dtype=dtype, lmin=1, lmax=300, seed=D + bs)
    _check(out, ref, dtype)
    assert b2pa.read_status(cuda_device) == 0


@pytest.mark.parametrize("H", [1, 2, 3, 6, 12])
def test_decode_head_groupings(cuda_device, H):
    out, ref = _random_decode(cuda_device, B=6, H=H, D=64, bs=16, dtype=torch.float32, lmin=1, lmax=700, seed=H)
    _check(out, ref, torch.float32)


def test_decode_edge_lengths(cuda_device):
    # empty sequence, block boundaries 1/15/16/17/32/33, cur_len 0 (sees all),
    # cur_len 2 (sees one fewer), cur_len > seq_len (sees nothing)
    lens = [0, 1, 15, 16, 17, 32, 33, 100, 5, 9]
    cur = [1, 1, 1, 1, 1, 1, 1, 0, 2, 20]
    out, ref = _random_decode(cuda_device, B=len(lens), H=4, D=64, bs=16, dtype=torch.float32, lmin=0, lmax=0,
                              seed=11, cur=cur, lens=lens)
    _check(out, ref, torch.float32)
    assert out[0].abs().sum().item() == 0 and out[9].abs().sum().item() == 0


def test_decode_many_sequences_plan(cuda_device):
    # more than 1024 sequences: the split planner scans in several chunks
    out, ref = _random_decode(cuda_device, B=2500, H=2, D=32, bs=16, dtype=torch.float32, lmin=0, lmax=90, seed=5)
    _check(out, ref, torch.float32)


def _many_stream_lengths(rng, B):
    """Mostly short contexts (zeros, block edges) plus three long ones, so
    that with B * H / 4 >= 444 head-group streams the contiguous split cuts
    streams between CTAs, some across many CTAs."""
    lens = rng.integers(0, 200, size=B)
    lens[:8] = [0, 1, 15, 16, 17, 32, 0, 33]
    lens[100], lens[700], lens[B - 1] = 9000, 16000, 12345
    return lens.tolist()


@pytest.mark.parametrize("dtype,D,bs", [(torch.bfloat16, 16, 16), (torch.float32, 32, 16), (torch.float16, 128, 16),
                                        (torch.bfloat16, 64, 8), (torch.float32, 64, 32)])
def test_decode_contiguous_split(cuda_device, dtype, D, bs):
    """2400 or more head-group streams: each CTA streams an equal range of
    pages and streams cut between CTAs are merged by the combine kernel;
    cur_len 0 / 2 / past the length included.  Two calls give the same
    bytes."""
    rng = np.random.default_rng(31)
    B, H = 1200, 8
    lens = _many_stream_lengths(rng, B)
    cur = [1] * B
    cur[3], cur[9], cur[700], cur[11] = 0, 2, 3, 500
    out, ref = _random_decode(cuda_device, B=B, H=H, D=D, bs=bs, dtype=dtype, lmin=0, lmax=0, seed=31, cur=cur,
                              lens=lens)
    _check(out, ref, dtype)
    assert out[6].abs().sum().item() == 0 and out[11].abs().sum().item() == 0
    again, _ = _random_decode(cuda_device, B=B, H=H, D=D, bs=bs, dtype=dtype, lmin=0, lmax=0, seed=31, cur=cur,
                              lens=lens)
    assert torch.equal(out, again)
    assert b2pa.read_status(cuda_device) == 0


def test_decode_contiguous_split_plan_kernel(cuda_device):
    """9,000 sequences: the unit offsets of the contiguous split come from the
    one-CTA plan launch (too many for each CTA's shared memory); empty
    sequences and a long one among them."""
    rng = np.random.default_rng(41)
    lens = rng.integers(0, 40, size=9000)
    lens[4500] = 5000
    out, ref = _random_decode(cuda_device, B=9000, H=1, D=64, bs=16, dtype=torch.float32, lmin=0, lmax=0, seed=41,
                              lens=lens.tolist())
    _check(out, ref, torch.float32)
    assert b2pa.read_status(cuda_device) == 0


def test_decode_contiguous_split_many_pieces(cuda_device):
    """A 20,000-token sequence among 511 short ones (1,024 head-group
    streams): with about 8 pages per CTA its streams are cut into well over
    32 pieces, which the combine kernel merges 32 at a time."""
    rng = np.random.default_rng(43)
    lens = rng.integers(0, 30, size=512)
    lens[200] = 20000
    out, ref = _random_decode(cuda_device, B=512, H=8, D=64, bs=16, dtype=torch.float32, lmin=0, lmax=0, seed=43,
                              lens=lens.tolist())
    _check(out, ref, torch.float32)
    assert b2pa.read_status(cuda_device) == 0


def test_decode_long_contexts_split(cuda_device):
    # few sequences, long contexts: many pages per sequence -> split-K + combine
    out, ref = _random_decode(cuda_device, B=3, H=8, D=128, bs=16, dtype=torch.bfloat16, lmin=4000, lmax=9000,
                              seed=6)
    _check(out, ref, torch.bfloat16)


def test_config1_decode_plus_append(cuda_device):
    """64 sequences, L ~ U[128,1024], H=8, D=64, fp32,
    4096-block pool, random non-overlapping tables; append 1 token then decode."""
    rng = np.random.default_rng(1)
    B, H, D, bs, NB = 64, 8, 64, 16, 4096
    lens0 = rng.integers(128, 1025, size=B).tolist()
    gen = torch.Generator().manual_seed(1)
    kp = torch.randn(NB, H, bs, D, generator=gen).to(cuda_device)
    vp = torch.randn(NB, H, bs, D, generator=gen).to(cuda_device)
    tables = random_tables(rng, lens0, NB, bs)
    cache = build_cache(b2pa, kp, vp, tables, lens0, bs)  # unused blocks form the free list
    k_new = strided_q(B, H, 1, D, torch.float32, cuda_device, gen)
    v_new = strided_q(B, H, 1, D, torch.float32, cuda_device, gen)
    q = strided_q(B, H, 1, D, torch.float32, cuda_device, gen)
    ret = cache.append_batch(k_new, v_new, 1)
    assert ret.tolist() == [L + 1 for L in lens0]
    out = b2pa.paged_attention("b200_paged", q, cache, 1)
    tables_now = [list(s.block_ids) for s in cache.states]
    kp_h, vp_h = kp.cpu().numpy(), vp.cpu().numpy()
    ref = orc.paged_attention_c(q.cpu().numpy(), kp_h, vp_h, tables_now, [L + 1 for L in lens0], [1] * B)
    _check(out, ref, torch.float32)
    # the appended token landed where the reference's allocator put it
    kn = k_new.cpu().numpy()
    for b, (st, L) in enumerate(zip(cache.states, lens0)):
        blk, off = st.block_ids[L // bs], L % bs
        assert np.array_equal(kp_h[blk, :, off, :].view(np.int32), kn[b, :, 0, :].view(np.int32))
    assert b2pa.read_status(cuda_device) == 0


def test_config4_subset(cuda_device):
    """BASELINE config[4] shape on a 12-sequence subset: H=32, D=128, bf16,
    L ~ U[1024, 8192], pool 1.2x the pages."""
    rng = np.random.default_rng(4)
    lens = rng.integers(1024, 8193, size=12).tolist()
    pages = sum(-(-L // 16) for L in lens)
    out, ref = _random_decode(cuda_device, B=12, H=32, D=128, bs=16, dtype=torch.bfloat16, lmin=0, lmax=0, seed=4,
                              lens=lens, nb_extra=int(0.2 * pages))
    _check(out, ref, torch.bfloat16)


def test_bad_block_id_is_reported(cuda_device):
    torch.manual_seed(0)
    kp = torch.randn(4, 2, 16, 64, device=cuda_device)
    vp = torch.randn_like(kp)
    cache = build_cache(b2pa, kp, vp, [[0, 9]], [20], 16)  # block 9 is past the pool
    b2pa.clear_status(cuda_device)
    q = torch.randn(1, 2, 1, 64, device=cuda_device)
    out = b2pa.paged_attention("b200_paged", q, cache, 1)
    assert b2pa.read_status(cuda_device) == -3
    b2pa.clear_status(cuda_device)
    assert torch.isfinite(out).all()


def test_decode_repeatable_and_stream_safe(cuda_device):
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out1, ref = _random_decode(cuda_device, B=33, H=8, D=128, bs=16, dtype=torch.bfloat16, lmin=1, lmax=2000,
                                   seed=9)
    s.synchronize()
    out2, _ = _random_decode(cuda_device, B=33, H=8, D=128, bs=16, dtype=torch.bfloat16, lmin=1, lmax=2000, seed=9)
    assert torch.equal(out1, out2)
    _check(out1, ref, torch.bfloat16)


def test_split_decode_reuses_workspace_and_replays_in_a_graph(cuda_device):
    """Split sequences go through the combine launch: repeated calls on one
    workspace and CUDA-graph replays of the kernel call give the oracle's
    output every time."""
    rng = np.random.default_rng(21)
    gen = torch.Generator().manual_seed(21)
    B, H, D, bs = 4, 8, 128, 16
    lens = rng.integers(3000, 7000, size=B).tolist()
    NB = sum(-(-L // bs) for L in lens) + 5
    kp = torch.randn(NB, H, bs, D, generator=gen).to(torch.bfloat16).to(cuda_device)
    vp = torch.randn(NB, H, bs, D, generator=gen).to(torch.bfloat16).to(cuda_device)
    tables = random_tables(rng, lens, NB, bs)
    cache = build_cache(b2pa, kp, vp, tables, lens, bs)
    q = strided_q(B, H, 1, D, torch.bfloat16, cuda_device, gen)
    ref = orc.paged_attention_c(q.float().cpu().numpy(), kp.float().cpu().numpy(), vp.float().cpu().numpy(), tables,
                                lens, [1] * B)
    from b2pa.paged_kv import device_metadata

    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(3):
            out = b2pa.paged_attention("b200_paged", q, cache, 1)
            _check(out, ref, torch.bfloat16)
        # capture the kernel call alone (metadata prepared outside the graph)
        table, seq_lens, max_pages = device_metadata(cache, torch.device(cuda_device))
        table = table[:, :max_pages]
        cur = torch.ones(B, dtype=torch.int32, device=cuda_device)
        out = b2pa.paged_attention_decode_b200(q, kp, vp, table, seq_lens, cur)
        _check(out, ref, torch.bfloat16)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            gout = b2pa.paged_attention_decode_b200(q, kp, vp, table, seq_lens, cur)
        for _ in range(3):
            gout.zero_()
            g.replay()
            s.synchronize()
            _check(gout, ref, torch.bfloat16)
    s.synchronize()
    del g
    assert b2pa.read_status(cuda_device) == 0
