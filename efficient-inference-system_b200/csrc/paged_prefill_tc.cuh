// paged_prefill_tc.cuh -- chunked-prefill paged attention on the 5th-gen
// tensor cores (tcgen05 + TMEM), bf16/fp16 inputs, fp32 accumulation.
//
// Replaces the Triton prefill kernel of the reference
// (src/kernels/triton_paged_attention.py:88-176, launcher :220-258) for
// 16-bit pools with head_dim 64 or 128; semantics as in
// src/kernels/reference_paged_attention.py:31-57 (query row t of sequence b
// sees keys 0 .. min(seq_len, seq_len - cur_len + t + 1) - 1; rows that see
// nothing are zero; rows past cur_len see the whole sequence).
//
// One CTA = (128 query rows, head, sequence); 6 warps:
//   warp 4  producer: per 64-key tile, one TMA tensor load per page and
//           128-byte column block for K and for V (block table gather; the
//           pool is viewed as a 2-d [blocks*H*block_size, D] tensor with a
//           128B-swizzle map), into a 2-stage ring;
//   warp 5  MMA issuer (one elected lane): S = Q.K^T (M=128, N=64, K=D) into
//           TMEM, then O_tile = P.V (M=128, N=D, K=64) into TMEM; completion
//           signalled with tcgen05.commit on mbarriers;
//   warps 0-3 softmax: thread r owns query row r: reads its S row from TMEM,
//           masks, online softmax in the log2 domain, writes P (bf16/fp16,
//           128B-swizzled K-major) to shared memory for the next MMA, and
//           accumulates O_tile from TMEM into fp32 registers with the
//           running rescale.  The output is divided by max(l, 1e-9).
// Q is loaded by the softmax threads (arbitrary strides) into the swizzled
// layout.  Every mbarrier wait is bounded (1 s); a wait that gives up records
// B2PA_ERR_DEVICE_TIMEOUT, raises a CTA-wide abort flag and the roles drain
// to the final barrier so TMEM is always freed.  No multicast anywhere.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace b2pa {

struct PfTcParams {
  const void* q;
  int64_t sq_b, sq_h, sq_t;
  const int32_t* page_table;
  int64_t pt_stride;
  int max_pages;
  const int32_t* seq_lens;
  const int32_t* cur_lens;
  void* out;
  int64_t so_b, so_h, so_t;
  int B, H, T;
  int64_t num_blocks;
  float scale_log2;
  int32_t* status;
  // Key-range split: CTA (x = q_tile * nsplit_max + s) covers key tiles
  // [s*kt_per_split, (s+1)*kt_per_split).  With more than one split the CTAs
  // write fp32 partials (unnormalised O, running max m, denominator l) that
  // prefill_combine_kernel merges.
  int kt_per_split;
  int nsplit_max;
  int max_cta_pages;  // capacity of the block-id array staged in shared memory
  float* part_o;   // [B, H, T, nsplit_max, D]
  float* part_ml;  // [B, H, T, nsplit_max, 2]
};

// Key tiles of query tile `t0` of sequence b, and its number of splits.
__device__ __forceinline__ void prefill_tile_range(const PfTcParams& p, int b, int t0, int bm, int bn, int bs,
                                                   int64_t* kend_out, int* ntiles_out, int* nsplit_out) {
  const int64_t L = p.seq_lens[b];
  const int64_t past = L - (int64_t)p.cur_lens[b];
  const int64_t cap = (int64_t)p.max_pages * bs;
  const int t_last = (t0 + bm < p.T ? t0 + bm : p.T) - 1;
  int64_t kend = L < past + t_last + 1 ? L : past + t_last + 1;
  if (kend > cap) kend = cap;
  if (kend < 0) kend = 0;
  const int ntiles = (int)((kend + bn - 1) / bn);
  const int ns = (ntiles + p.kt_per_split - 1) / p.kt_per_split;
  *kend_out = kend;
  *ntiles_out = ntiles;
  *nsplit_out = ns < 1 ? 1 : ns;
}

template <int D, int BS>
struct PfTcCfg {
  static constexpr int BM = 128;         // query rows per CTA (UMMA M)
  static constexpr int BN = 64;          // keys per tile
  static constexpr int KB = D / 64;      // 128-byte column blocks of a row
  static constexpr int PAGES = BN / BS;  // pages per key tile
  // K/V ring depth: a stage is refilled only after the P.V MMA that read it,
  // so the load of tile j+STAGES overlaps the softmax of STAGES tiles.
  static constexpr int STAGES = D == 64 ? 6 : 4;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int P_BYTES = BM * BN * 2;  // one P buffer; two are kept
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_P = OFF_V + STAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
  // kv_full[STAGES], kv_empty[STAGES], s_full[2], p_full[2], o_full[2]
  static constexpr int N_BARS = 2 * STAGES + 6;
  static constexpr int OFF_MISC = OFF_BAR + 8 * N_BARS;
  static constexpr int OFF_BLK = OFF_MISC + 16;      // int32 block ids of the CTA's pages
  static constexpr int SMEM_FIXED = OFF_BLK + 1024;  // + alignment slack; + 4 * max_cta_pages
  // TMEM: S[2] (BN columns each) then the O accumulator (D columns).
  static constexpr int TMEM_USED = 2 * BN + D;
  static constexpr int TMEM_COLS = TMEM_USED <= 256 ? 256 : 512;
  static constexpr int MIN_BLOCKS = 1;
  static constexpr int THREADS = 192;
  static_assert(D == 64 || D == 128, "tcgen05 prefill is built for head_dim 64 and 128");
  static_assert(BN % BS == 0, "block size must divide the key tile");
};

// Waits with every lane of the warp; false (for all lanes) if any gave up.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int32_t* status, volatile int* abort_flag) {
  if (*abort_flag) return false;
  const bool ok = __all_sync(kFullMask, mbar_wait_bounded(bar, parity, status));
  if (!ok) *abort_flag = 1;
  return ok;
}

template <typename T, int D, int BS>
__global__ void __launch_bounds__(192, PfTcCfg<D, BS>::MIN_BLOCKS)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            PfTcParams p) {
  using C = PfTcCfg<D, BS>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = smem + C::OFF_Q;
  unsigned char* sK = smem + C::OFF_K;
  unsigned char* sV = smem + C::OFF_V;
  unsigned char* sP = smem + C::OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + C::STAGES;
  uint64_t* s_full = bars + 2 * C::STAGES;  // [2]
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* o_full = s_full + 4;            // one phase per P.V MMA
  uint64_t* o_final = s_full + 5;           // one phase: every P.V of the CTA done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  int* sblk = reinterpret_cast<int*>(smem + C::OFF_BLK);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x % p.nsplit_max;
  const int t0 = (blockIdx.x / p.nsplit_max) * C::BM;
  const int h = blockIdx.y;
  const int b = blockIdx.z;

  const int64_t L = p.seq_lens[b];
  const int64_t past = L - (int64_t)p.cur_lens[b];
  const int64_t cap = (int64_t)p.max_pages * BS;
  int64_t kend;
  int ntiles_all, nsplit;
  prefill_tile_range(p, b, t0, C::BM, C::BN, BS, &kend, &ntiles_all, &nsplit);
  if (split >= nsplit) return;  // this query tile needs fewer splits (uniform across the CTA)
  const int j0 = split * p.kt_per_split;
  const int j1 = (j0 + p.kt_per_split < ntiles_all) ? j0 + p.kt_per_split : ntiles_all;
  const int ntiles = j1 > j0 ? j1 - j0 : 0;  // tiles of this CTA; tile index = j0 + local

  if (tid == 0) {
    if (L > cap) set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    tc::prefetch_tmap(&tm_k);
    tc::prefetch_tmap(&tm_v);
  }
  {
    // Block ids of this CTA's pages, validated once: -1 for pages past the
    // visible range or with an id outside the pool (reported).
    const int64_t pg0 = (int64_t)j0 * C::PAGES;
    const int npg = ntiles * C::PAGES;
    for (int i = tid; i < npg; i += C::THREADS) {
      const int64_t page = pg0 + i;
      int blk = -1;
      if (page * BS < kend) {
        blk = p.page_table[(int64_t)b * p.pt_stride + page];
        if (blk >= p.num_blocks) {
          set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
          blk = -1;
        }
      }
      sblk[i] = blk;
    }
  }
  if (warp < 4) {
    // Q rows -> 128B-swizzled K-major tile, zeros past T.
    const int r = tid;
    const int t = t0 + r;
    const T* qrow = static_cast<const T*>(p.q) + (int64_t)b * p.sq_b + (int64_t)h * p.sq_h + (int64_t)t * p.sq_t;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t < p.T) v = *reinterpret_cast<const uint4*>(qrow + c * 8);
      *reinterpret_cast<uint4*>(sQ + (c >> 3) * (C::BM * 128) + tc::sw128_offset(r, c & 7)) = v;
    }
    tc::fence_proxy_async_smem();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // S(j) in columns [ (j%2)*BN, +BN ); O accumulates in [ 2*BN, 2*BN + D ).
  const uint32_t tS0 = tmem;
  const uint32_t tO = tmem + 2 * C::BN;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % C::STAGES;
      const uint32_t ph = (uint32_t)(j / C::STAGES) & 1u;
      if (!warp_wait(&kv_empty[st], ph ^ 1u, p.status, abort_flag)) break;
      int blks[C::PAGES];
      uint32_t bytes = 0;
#pragma unroll
      for (int pg = 0; pg < C::PAGES; ++pg) {
        const int blk = sblk[j * C::PAGES + pg];
        blks[pg] = blk;
        if (blk >= 0) {
          bytes += 2u * BS * D * 2;
        } else {
          // Pages that are not loaded must not hold stale or uninitialised
          // bytes: their softmax weight is 0, but 0 * NaN is NaN in P.V.
#pragma unroll
          for (int kb = 0; kb < C::KB; ++kb) {
            const int off = st * C::KV_BYTES + kb * (C::BN * 128) + pg * (BS * 128);
            for (int i = lane; i < BS * 8; i += 32) {
              reinterpret_cast<uint4*>(sK + off)[i] = make_uint4(0, 0, 0, 0);
              reinterpret_cast<uint4*>(sV + off)[i] = make_uint4(0, 0, 0, 0);
            }
          }
        }
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&kv_full[st], bytes);
#pragma unroll
        for (int pg = 0; pg < C::PAGES; ++pg) {
          if (blks[pg] < 0) continue;
          const int row = (blks[pg] * p.H + h) * BS;
#pragma unroll
          for (int kb = 0; kb < C::KB; ++kb) {
            const int off = st * C::KV_BYTES + kb * (C::BN * 128) + pg * (BS * 128);
            tc::tma_load_2d(sK + off, &tm_k, kb * 64, row, &kv_full[st]);
            tc::tma_load_2d(sV + off, &tm_v, kb * 64, row, &kv_full[st]);
          }
        }
      }
      __syncwarp();
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issue
    // Order: QK(0), QK(1), then per tile j: PV(j) once P(j) is ready, then
    // QK(j+2) into the S buffer tile j just released.  The softmax of tile
    // j+1 therefore overlaps PV(j) and the load of tile j+2.
    constexpr int FMT = sizeof(T) == 2 && ElemTraits<T>::kDtype == B2PA_DTYPE_BF16 ? 1 : 0;
    constexpr uint32_t idesc_s = tc::idesc_f16(128, C::BN, FMT, 0, 0);
    constexpr uint32_t idesc_o = tc::idesc_f16(128, D, FMT, 0, 1);
    const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
    auto issue_qk = [&](int j) -> bool {
      const int st = j % C::STAGES;
      if (!warp_wait(&kv_full[st], (uint32_t)(j / C::STAGES) & 1u, p.status, abort_flag)) return false;
      tc::fence_after_sync();
      if (lane == 0) {
        const uint32_t tS = tS0 + (uint32_t)(j & 1) * C::BN;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int kb = k >> 2, kk = k & 3;
          const uint64_t a = tc::smem_desc(aQ + kb * (C::BM * 128) + kk * 32, 16, 1024);
          const uint64_t bd = tc::smem_desc(aK + st * C::KV_BYTES + kb * (C::BN * 128) + kk * 32, 16, 1024);
          tc::mma_f16_ss(tS, a, bd, idesc_s, k > 0);
        }
        tc::commit(&s_full[j & 1]);
      }
      __syncwarp();
      return true;
    };
    bool ok = true;
    if (ntiles > 0) ok = issue_qk(0);
    if (ok && ntiles > 1) ok = issue_qk(1);
    for (int j = 0; j < ntiles && ok; ++j) {
      const int st = j % C::STAGES;
      if (!warp_wait(&p_full[j & 1], (uint32_t)(j >> 1) & 1u, p.status, abort_flag)) break;
      tc::fence_after_sync();
      if (lane == 0) {
        const uint32_t aPj = aP + (uint32_t)(j & 1) * C::P_BYTES;
#pragma unroll
        for (int k = 0; k < C::BN / 16; ++k) {
          const uint64_t a = tc::smem_desc(aPj + k * 32, 16, 1024);
          const uint64_t bd = tc::smem_desc(aV + st * C::KV_BYTES + k * 2048, C::BN * 128, 1024);
          tc::mma_f16_ss(tO, a, bd, idesc_o, j > 0 || k > 0);
        }
        tc::commit(o_full);
        tc::commit(&kv_empty[st]);
      }
      __syncwarp();
      if (j + 2 < ntiles) ok = issue_qk(j + 2);
    }
    // The epilogue cannot wait on o_full by parity: when it runs, only
    // P.V(ntiles-3) is known complete, so o_full may still be two phases
    // behind.  A separate single-phase barrier marks "all MMAs done".
    if (ok && ntiles > 0 && lane == 0) tc::commit(o_final);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int r = tid;
    const int t = t0 + r;
    int64_t row_end = L < past + t + 1 ? L : past + t + 1;
    if (row_end > cap) row_end = cap;
    const uint32_t trow = (uint32_t)(warp * 32) << 16;
    // O accumulates in TMEM at the scale 2^m_ref.  m_ref only moves when a
    // tile's row max exceeds it by more than kRescale (log2 units), so the
    // P values stay below 2^kRescale and the rescale of O (TMEM load, scale,
    // store) is rare.  Rescaling at tile j waits for P.V(j-1): the o_full
    // barrier completes one phase per P.V; S(j) being ready implies every MMA
    // issued before QK(j) -- so P.V(j-2) -- is done, and P.V(j) cannot start
    // before this warp releases P(j), so o_full is in phase j-1 or j and the
    // parity wait is exact.
    constexpr float kRescale = 8.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (!warp_wait(&s_full[j & 1], (uint32_t)(j >> 1) & 1u, p.status, abort_flag)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      float s[64];
      {
        const uint32_t tS = tS0 + (uint32_t)(j & 1) * C::BN;
        float a[32], c[32];
        tc::tmem_ld32(tS + trow, a);
        tc::tmem_ld32(tS + trow + 32, c);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = a[i];
          s[32 + i] = c[i];
        }
      }
      const int64_t k0 = (int64_t)(j0 + j) * C::BN;
      bool all_pages = true;
      bool page_ok[C::PAGES];
#pragma unroll
      for (int pg = 0; pg < C::PAGES; ++pg) {
        page_ok[pg] = sblk[j * C::PAGES + pg] >= 0;
        all_pages = all_pages && page_ok[pg];
      }
      // Keys of this tile visible to this row: [0, lim) (and pages present).
      const int64_t lim64 = row_end - k0;
      const int lim = lim64 < 0 ? 0 : (lim64 > C::BN ? C::BN : (int)lim64);
      if (lim == C::BN && all_pages) {
#pragma unroll
        for (int i = 0; i < 64; ++i) s[i] *= p.scale_log2;
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const bool vis = i < lim && page_ok[i / BS];
          s[i] = vis ? s[i] * p.scale_log2 : -INFINITY;
        }
      }
      // Row max as a tree (short dependency chains: one warp per SM
      // sub-partition runs this, so latency, not throughput, bounds it).
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = fmaxf(fmaxf(s[i], s[i + 8]), fmaxf(s[i + 16], s[i + 24]));
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = fmaxf(mx[i], fmaxf(fmaxf(s[i + 32], s[i + 40]), fmaxf(s[i + 48], s[i + 56])));
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      // A row moves its reference max when the tile's max exceeds it by more
      // than kRescale.  Rows that already hold O at the old scale need O and
      // l multiplied by 2^(m_old - m_new); a row with no visible key so far
      // (m = -inf) holds zeros and just adopts the new max.  TMEM accesses
      // and the barrier wait are warp-collective, so the whole warp takes
      // the branch if any lane needs it (other lanes scale by 1).
      const bool need = mt > m + kRescale;
      const float m_new = need ? mt : m;
      const bool scale_o = need && m != -INFINITY;
      if (j > 0 && __any_sync(kFullMask, scale_o)) {
        const float alpha = scale_o ? fast_exp2(m - m_new) : 1.f;
        // wait for P.V(j-1) before touching O
        if (!warp_wait(o_full, (uint32_t)(j - 1) & 1u, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int cb = 0; cb < D / 32; ++cb) {
          float ov[32];
          tc::tmem_ld32(tO + trow + cb * 32, ov);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= alpha;
          tc::tmem_st32(tO + trow + cb * 32, ov);
        }
        tc::tmem_wait_st();
        l *= alpha;
      }
      m = m_new;
      const bool live = m != -INFINITY;
      float ls[8];  // 8 independent partial sums
#pragma unroll
      for (int e = 0; e < 8; ++e) ls[e] = 0.f;
      unsigned char* sPj = sP + (j & 1) * C::P_BYTES;  // free: S(j) ready implies P.V(j-2) done
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pv[e] = live ? fast_exp2(s[c8 * 8 + e] - m) : 0.f;
          ls[e] += pv[e];
        }
        Vec<T, 8> w;
        w.from_float(pv);
        *reinterpret_cast<uint4*>(sPj + tc::sw128_offset(r, c8)) = w.w;
      }
      l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j & 1]);
    }
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.f;
    if (ok && ntiles > 0 && warp_wait(o_final, 0u, p.status, abort_flag)) {
      tc::fence_after_sync();
#pragma unroll
      for (int cb = 0; cb < D / 32; ++cb) tc::tmem_ld32(tO + trow + cb * 32, *reinterpret_cast<float(*)[32]>(o + cb * 32));
      tc::tmem_wait_ld();
    }
    tc::fence_before_sync();
    if (t < p.T && nsplit > 1) {
      const int64_t slot = (((int64_t)b * p.H + h) * p.T + t) * p.nsplit_max + split;
      float4* po = reinterpret_cast<float4*>(p.part_o + slot * D);
#pragma unroll
      for (int c4 = 0; c4 < D / 4; ++c4) po[c4] = make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]);
      p.part_ml[2 * slot] = m;
      p.part_ml[2 * slot + 1] = l;
    } else if (t < p.T) {
      const float den = fmaxf(l, 1e-9f);
      T* orow = static_cast<T*>(p.out) + (int64_t)b * p.so_b + (int64_t)h * p.so_h + (int64_t)t * p.so_t;
#pragma unroll
      for (int c8 = 0; c8 < D / 8; ++c8) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = o[c8 * 8 + e] / den;
        Vec<T, 8> w;
        w.from_float(f);
        *reinterpret_cast<uint4*>(orow + c8 * 8) = w.w;
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// One warp per (sequence, head, query row) whose query tile was split:
// log-sum-exp merge of the split partials, then the reference's normalisation.
template <typename T, int D, int BS>
__global__ void __launch_bounds__(256) prefill_combine_kernel(PfTcParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= (int64_t)p.B * p.H * p.T) return;
  const int t = (int)(row % p.T);
  const int h = (int)((row / p.T) % p.H);
  const int b = (int)(row / ((int64_t)p.T * p.H));
  int64_t kend;
  int ntiles, nsplit;
  prefill_tile_range(p, b, (t / 128) * 128, 128, 64, BS, &kend, &ntiles, &nsplit);
  if (nsplit <= 1) return;
  const int64_t base = row * p.nsplit_max;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, p.part_ml[2 * (base + s)]);
  constexpr int PER = D / 32;
  float o[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) o[i] = 0.f;
  float L = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float ms = p.part_ml[2 * (base + s)];
    const float w = (M == -INFINITY) ? 0.f : exp2f(ms - M);
    L = fmaf(p.part_ml[2 * (base + s) + 1], w, L);
    const float* po = p.part_o + (base + s) * D;
#pragma unroll
    for (int i = 0; i < PER; ++i) o[i] = fmaf(w, po[lane + 32 * i], o[i]);
  }
  const float den = fmaxf(L, 1e-9f);
  T* orow = static_cast<T*>(p.out) + (int64_t)b * p.so_b + (int64_t)h * p.so_h + (int64_t)t * p.so_t;
#pragma unroll
  for (int i = 0; i < PER; ++i) orow[lane + 32 * i] = from_f32<T>(o[i] / den);
}

// ----------------------------------------------------------------- host ---
bool encode_pool_tensor_map(CUtensorMap* map, const void* pool, int64_t rows, int D, int block_size, int dtype);

template <typename T, int D, int BS>
int launch_prefill_tc(const AttnArgs& a, cudaStream_t stream) {
  using C = PfTcCfg<D, BS>;
  CUtensorMap tmk, tmv;
  const int64_t rows = a.num_blocks * a.H * BS;
  if (!encode_pool_tensor_map(&tmk, a.k_pool, rows, D, BS, a.dtype) ||
      !encode_pool_tensor_map(&tmv, a.v_pool, rows, D, BS, a.dtype))
    return set_error(B2PA_ERR_CUDA, "paged_prefill: cuTensorMapEncodeTiled failed for the pools");
  PfTcParams p;
  p.q = a.q;
  p.sq_b = a.sq[0];
  p.sq_h = a.sq[1];
  p.sq_t = a.sq[2];
  p.page_table = a.page_table;
  p.pt_stride = a.pt_stride;
  p.max_pages = a.max_pages;
  p.seq_lens = a.seq_lens;
  p.cur_lens = a.cur_lens;
  p.out = a.out;
  p.so_b = a.so[0];
  p.so_h = a.so[1];
  p.so_t = a.so[2];
  p.B = a.B;
  p.H = a.H;
  p.T = a.T;
  p.num_blocks = a.num_blocks;
  p.scale_log2 = a.scale * kLog2e;
  p.status = a.status;
  const PrefillPlan plan = make_prefill_plan(a.B, a.H, a.T, a.D, a.max_pages, BS, a.dtype);
  p.kt_per_split = plan.kt_per_split;
  p.nsplit_max = plan.nsplit_max;
  p.part_o = nullptr;
  p.part_ml = nullptr;
  if (plan.bytes > 0) {
    if (!a.workspace || a.workspace_bytes < plan.bytes)
      return set_error(B2PA_ERR_WORKSPACE, "paged_prefill: workspace of %zu bytes, %zu needed", a.workspace_bytes,
                       plan.bytes);
    p.part_ml = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + plan.off_part_ml);
    p.part_o = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + plan.off_part_o);
  }
  const int64_t ktmax = ((int64_t)a.max_pages * BS + C::BN - 1) / C::BN;
  const int64_t kt_cta = plan.nsplit_max > 1 ? plan.kt_per_split : ktmax;
  p.max_cta_pages = (int)((kt_cta > 0 ? kt_cta : 1) * C::PAGES);
  const size_t smem = C::SMEM_FIXED + 4 * (size_t)p.max_cta_pages;
  if (smem > (size_t)device_max_smem_optin())
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_prefill: %d pages per CTA exceed shared memory", p.max_cta_pages);
  auto kern = paged_prefill_tc_kernel<T, D, BS>;
  int rc_attr = set_max_dynamic_smem_cached(reinterpret_cast<const void*>(kern), (int)smem);
  if (rc_attr != B2PA_OK) return rc_attr;
  cudaError_t e;
  dim3 grid(((a.T + C::BM - 1) / C::BM) * plan.nsplit_max, a.H, a.B);
  kern<<<grid, C::THREADS, smem, stream>>>(tmk, tmv, p);
  if (plan.nsplit_max > 1) {
    const int64_t rows = (int64_t)a.B * a.H * a.T;
    prefill_combine_kernel<T, D, BS><<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(p);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_prefill_tc launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

}  // namespace b2pa
