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
// One CTA = (128 query rows, head, sequence); NG softmax warpgroups (two for
// head_dim 64, one for 128) plus three warps:
//   K and V producer warps: per 64-key tile, one TMA tensor load per page and
//           128-byte column block (block-table gather; the pool is viewed as a
//           2-d [blocks*H*block_size, D] tensor with a 128B-swizzle map) into
//           a STAGES-deep K ring and a STAGES-deep V ring.  A K stage is
//           refilled as soon as its Q.K^T is done, well before the P.V of
//           the same tile frees its V stage.  They read block ids straight
//           from the table, so the first loads leave before the rest of the
//           CTA has finished setting up;
//   two MMA issuer warps (one elected lane each): the QK warp issues
//           S = Q.K^T (M=128, N=64, K=D) into TMEM up to NSLOT tiles ahead of
//           the softmax; the PV warp issues O_g += P.V (M=128, N=D, K=64)
//           into the TMEM accumulator of the tile's group.  Splitting the
//           issue halves the serial chain of waits, MMAs and commits per tile
//           on each issuer; hand-overs go through mbarriers (tcgen05.commit);
//   softmax warpgroups: key tile j belongs to group j % NG; thread r of a
//           group owns query row r: reads its S row from TMEM, masks, online
//           softmax in the log2 domain, writes P (bf16/fp16, 128B-swizzled
//           K-major) to shared memory for the P.V MMA, and rescales its O in
//           TMEM when its running max moves by more than 2^8.  The epilogue
//           merges the groups' (max, denominator, O) and divides by
//           max(l, 1e-9).
// Q is loaded by the softmax threads (arbitrary strides) into the swizzled
// layout.  Every mbarrier wait is bounded (1 s); a wait that gives up records
// B2PA_ERR_DEVICE_TIMEOUT, raises a CTA-wide abort flag and the roles drain
// to the final barrier so TMEM is always freed.  No multicast anywhere.
#pragma once

#include <cuda.h>

#include <type_traits>

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
  int bm;             // query rows per CTA of the kernel that wrote the partials
  float* part_o;   // [B, H, T, nsplit_max, D]
  float* part_ml;  // [B, H, T, nsplit_max, 2]
  // fp32 variant: set to `epoch` (a number of this call) when an input lies
  // outside the range the fp16 hi/lo split represents; the kernel then stops,
  // and the fp32 CUDA-core kernel launched after it recomputes the call.
  // Marking with the call's number needs no reset between calls.
  uint32_t* range_flag;
  uint32_t epoch;
  // 1: the kernel before this one is b2pa's append kernel (see
  // AttnArgs::after_append): only the K/V producers wait for it, before
  // their first page copy; set-up, q and the block table go ahead.
  int early;
  // 1: Q is loaded by one TMA box per 64 columns (16-bit q whose layout the
  // tensor map takes); q_dim[0..2]: the map dimension of t, h, b.  0: the
  // softmax threads load it.
  int q_tma;
  int q_dim[3];
};

// Inputs of the fp32 variant must stay below 2^15 in magnitude (fp16 holds
// up to 65504; the lo part and the fp32 accumulations then stay in range).
// NaN and infinities fail the test too, so the CUDA-core kernel sees them.
constexpr float kSplitRange = 32768.f;

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

// SPLIT: the fp32 variant.  Every fp32 operand x (q, the K/V pages, P) is
// carried as two fp16 tiles, hi = fp16(x) and lo = fp16(x - hi), which
// together hold 22 significant bits, and each product is taken as
// hi*hi + hi*lo + lo*hi on the fp16 tensor cores with fp32 accumulation (the
// dropped lo*lo and the residual are ~2^-21 of the product).  A bf16 split
// (16 bits) was built first and missed the fp32 tolerance (atol 1e-5) on a
// few elements; fp16 meets it, but only holds |x| < 65504, so inputs at or
// above 2^15 (or not finite) raise range_flag and the call is recomputed by
// the general fp32 CUDA-core kernel, launched after this one as a backup that
// does nothing otherwise.  The K/V pages are split into a workspace copy
// beforehand (prefill_split_pages_kernel); q and P are split in the kernel.
template <int D, int BS, bool SPLIT = false>
struct PfTcCfg {
  static constexpr int BM = 128;         // query rows per CTA (UMMA M)
  static constexpr int BN = 64;          // keys per tile
  static constexpr int KB = D / 64;      // 128-byte column blocks of a row
  static constexpr int PAGES = BN / BS;  // pages per key tile
  static constexpr int NOP = SPLIT ? 2 : 1;  // bf16 tiles per operand tile (hi, lo)
  // Softmax warpgroups.  With two, key tiles alternate between them (tile j
  // -> group j % NG) and each keeps its own running max, denominator and O
  // accumulator; the groups are merged in the epilogue.  Two groups put two
  // softmax warps on every SM sub-partition, so one warp's exponentials
  // overlap the other's TMEM loads, barrier waits and P stores.
  static constexpr int NG = D == 64 ? 2 : 1;
  // S/P buffers: two per group; one per group for the fp32 variant, whose
  // hi/lo operand tiles take twice the shared memory (its two groups still
  // alternate, so one group's softmax overlaps the other's Q.K^T).
  static constexpr int NSLOT = SPLIT ? NG : 2 * NG;
  // Depth of the K ring and of the V ring.  A K stage is refilled once the
  // Q.K^T that read it is done, a V stage once its P.V is done, so each ring
  // loads up to STAGES tiles ahead of its consumer.
  static constexpr int STAGES = SPLIT ? 3 : (D == 64 ? 6 : 4);
  static constexpr int Q_TILE = BM * D * 2;   // one bf16 / fp16 tile
  static constexpr int KV_TILE = BN * D * 2;
  static constexpr int P_TILE = BM * BN * 2;
  static constexpr int Q_BYTES = NOP * Q_TILE;  // hi tile, then lo tile
  static constexpr int KV_BYTES = NOP * KV_TILE;
  static constexpr int P_BYTES = NOP * P_TILE;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_P = OFF_V + STAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + NSLOT * P_BYTES;
  // k_full, k_empty, v_full, v_empty [STAGES each], s_full, p_full, p_free [NSLOT each], o_full[NG], o_final,
  // q_full
  static constexpr int N_BARS = 4 * STAGES + 3 * NSLOT + NG + 2;
  static constexpr int OFF_MISC = OFF_BAR + 8 * N_BARS;  // TMEM base, abort flag
  static constexpr int OFF_ML = OFF_MISC + 16;           // per-group (m, l) of every row, for the merge
  static constexpr int OFF_BLK = OFF_ML + (NG > 1 ? 2 * NG * BM * 4 : 0);  // int32 block ids of the CTA's pages
  static constexpr int SMEM_FIXED = OFF_BLK + 1024;  // + alignment slack; + 4 * max_cta_pages
  // TMEM: S[NSLOT] (BN columns each), then one O accumulator per group.
  static constexpr int TMEM_USED = NSLOT * BN + NG * D;
  static constexpr int TMEM_COLS = TMEM_USED <= 256 ? 256 : 512;
  static constexpr int SOFTMAX_THREADS = 128 * NG;
  static constexpr int K_WARP = 4 * NG;       // K producer (also initialises the barriers)
  static constexpr int V_WARP = 4 * NG + 1;   // V producer
  static constexpr int QK_WARP = 4 * NG + 2;  // issues S = Q.K^T; owns the TMEM allocation
  static constexpr int PV_WARP = 4 * NG + 3;  // issues O += P.V
  static constexpr int THREADS = SOFTMAX_THREADS + 128;
  static_assert(D == 64 || D == 128, "tcgen05 prefill is built for head_dim 64 and 128");
  static_assert(!SPLIT || D == 64, "the fp32 variant fits shared memory for head_dim 64 only");
  static_assert(BN % BS == 0 && 32 % PAGES == 0, "block size must divide the key tile");
  static_assert(TMEM_USED <= 512, "TMEM holds 512 columns");
  static_assert(SMEM_FIXED <= 200 * 1024, "shared-memory plan");
};

// Named barriers (id 0 is __syncthreads): 1 = set-up done (every thread; the
// producer only arrives), 2 = softmax threads.
__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Wait by a single thread (the MMA issuer): the abort flag is read only while
// the barrier is not yet complete.  Gives up after kWaitLimitNs, records
// B2PA_ERR_DEVICE_TIMEOUT and raises the abort flag.
__device__ __forceinline__ bool lane_wait(uint64_t* bar, uint32_t parity, int32_t* status, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      set_status(status, B2PA_ERR_DEVICE_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
  }
}

// Waits with every lane of the warp; false (for all lanes) if any gave up.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int32_t* status, volatile int* abort_flag) {
  if (*abort_flag) return false;
  const bool ok = __all_sync(kFullMask, mbar_wait_bounded(bar, parity, status));
  if (!ok) *abort_flag = 1;
  return ok;
}

// Block id of local page `i` of a CTA (page pg0 + i of sequence b): -1 when
// past the keys the CTA reads or past the table; ids outside the pool are
// reported and read as -1.  `raw` is the table entry (loaded early).
__device__ __forceinline__ int prefill_checked_block(const PfTcParams& p, int raw, int64_t page, int64_t kend, int bs) {
  if (page >= p.max_pages || page * bs >= kend) return -1;
  if (raw >= p.num_blocks) {
    set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
    return -1;
  }
  return raw;
}

// fp32 pools take the split (fp16 hi/lo) variant of the kernel.
template <typename T>
constexpr bool kPfSplit = std::is_same<T, float>::value;

// Eight fp32 values as two 16-byte words of fp16: hi = round(x), lo =
// round(x - hi) (element 0 in the lowest bytes, as the tiles store them).
__device__ __forceinline__ void split_f16x8(const float (&f)[8], uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 hh = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    // x - hi as one packed fma with -1 (exact: the same bits as x - hi)
    const float2 r = fma2(__half22float2(hh), make_float2(-1.f, -1.f), make_float2(f[2 * i], f[2 * i + 1]));
    const __half2 ll = __floats2half2_rn(r.x, r.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&hh);
    l[i] = *reinterpret_cast<const uint32_t*>(&ll);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <typename T, int D, int BS>
__global__ void __launch_bounds__(PfTcCfg<D, BS, kPfSplit<T>>::THREADS, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const __grid_constant__ CUtensorMap tm_q, PfTcParams p) {
  constexpr bool SPLIT = kPfSplit<T>;
  using C = PfTcCfg<D, BS, SPLIT>;
  constexpr int NG = C::NG, NSLOT = C::NSLOT;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = smem + C::OFF_Q;
  unsigned char* sK = smem + C::OFF_K;
  unsigned char* sV = smem + C::OFF_V;
  unsigned char* sP = smem + C::OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* k_full = bars;
  uint64_t* k_empty = bars + C::STAGES;
  uint64_t* v_full = bars + 2 * C::STAGES;
  uint64_t* v_empty = bars + 3 * C::STAGES;
  uint64_t* s_full = bars + 4 * C::STAGES;  // [NSLOT]
  uint64_t* p_full = s_full + NSLOT;        // [NSLOT]: P(j) written (S(j) consumed)
  uint64_t* p_free = p_full + NSLOT;        // [NSLOT]: P.V(j) done, P buffer free
  uint64_t* o_full = p_free + NSLOT;        // [NG]: one phase per P.V MMA of the group
  uint64_t* o_final = o_full + NG;          // one phase: every P.V of the CTA done
  uint64_t* q_full = o_final + 1;           // one phase: Q landed (TMA load of Q only)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  float* sML = reinterpret_cast<float*>(smem + C::OFF_ML);
  int* sblk = reinterpret_cast<int*>(smem + C::OFF_BLK);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x % p.nsplit_max;
  const int t0 = (blockIdx.x / p.nsplit_max) * C::BM;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  // Q rows -> 128B-swizzled K-major tile, zeros past T, by the softmax
  // threads (the fp32 variant: hi tile, then lo tile, with the range check);
  // consecutive threads read consecutive 16-byte pieces of a row.
  auto load_q_threads = [&]() {
#pragma unroll
    for (int it = 0; it < C::BM * D / 8 / C::SOFTMAX_THREADS; ++it) {
      const int c = tid + it * C::SOFTMAX_THREADS;
      const int qr = c / (D / 8), qc = c % (D / 8);
      const int qt = t0 + qr;
      const int off = (qc >> 3) * (C::BM * 128) + tc::sw128_offset(qr, qc & 7);
      if constexpr (SPLIT) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = 0.f;
        if (qt < p.T) {
          const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.q) + (int64_t)b * p.sq_b +
                                                              (int64_t)h * p.sq_h + (int64_t)qt * p.sq_t + qc * 8);
          const float4 x0 = src[0], x1 = src[1];
          f[0] = x0.x; f[1] = x0.y; f[2] = x0.z; f[3] = x0.w;
          f[4] = x1.x; f[5] = x1.y; f[6] = x1.z; f[7] = x1.w;
          bool in_range = true;
#pragma unroll
          for (int e = 0; e < 8; ++e) in_range = in_range && fabsf(f[e]) < kSplitRange;
          if (!in_range) *p.range_flag = p.epoch;
        }
        uint4 hi, lo;
        split_f16x8(f, hi, lo);
        *reinterpret_cast<uint4*>(sQ + off) = hi;
        *reinterpret_cast<uint4*>(sQ + C::Q_TILE + off) = lo;
      } else {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (qt < p.T)
          v = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + (int64_t)b * p.sq_b +
                                              (int64_t)h * p.sq_h + (int64_t)qt * p.sq_t + qc * 8);
        *reinterpret_cast<uint4*>(sQ + off) = v;
      }
    }
  };
  // The fp32 variant's q is not written by its pre-pass: the softmax threads
  // split it while the pre-pass still runs.
  if constexpr (SPLIT) {
    if (tid < C::SOFTMAX_THREADS) load_q_threads();
  }
  // Launched programmatically after the kernel before it (the KV append of
  // the step, or the fp32 variant's pre-pass): wait for its results before
  // reading anything (after the append kernel, only before reading pool
  // pages: see PfTcParams::early); let the next kernel launch behind this grid.
  if (!p.early) pdl_wait();
  pdl_launch_dependents();
  if constexpr (SPLIT) {
    // an input out of the split's range was seen (pre-pass or another CTA):
    // the CUDA-core kernel that follows recomputes the call.  One read,
    // shared, so the whole CTA takes the same branch.
    __shared__ int stop;
    if (tid == 0) stop = *reinterpret_cast<volatile uint32_t*>(p.range_flag) == p.epoch;
    __syncthreads();
    if (stop) return;
  }
  const int j0 = split * p.kt_per_split;
  const int64_t pg0 = (int64_t)j0 * C::PAGES;
  const int32_t* pt_row = p.page_table + (int64_t)b * p.pt_stride;

  // Table entries of the first pages, read before the sequence length is
  // known so that both loads are in flight together (the producer: one page
  // per lane; the softmax threads: one page each, staged below).
  int blk_pre = -1;
  {
    const int i = warp == C::K_WARP || warp == C::V_WARP ? lane : tid;
    if (warp != C::QK_WARP && warp != C::PV_WARP && pg0 + i < p.max_pages) blk_pre = pt_row[pg0 + i];
  }

  // The K producer's lane 0 initialises the barriers at once and, when no
  // CTA of the launch can leave early (no key-range split), issues the TMA
  // load of Q before the sequence length is even known; otherwise once the
  // CTA is known to stay.  The QK issuer waits for it in every case.
  const bool q_first = p.q_tma && p.nsplit_max == 1;
  auto issue_q = [&]() {
    mbar_arrive_expect_tx(q_full, (uint32_t)C::Q_BYTES);
    auto coord = [&](int d) { return p.q_dim[0] == d ? t0 : (p.q_dim[1] == d ? h : b); };
#pragma unroll
    for (int kb = 0; kb < C::KB; ++kb)
      tc::tma_load_4d(sQ + kb * (C::BM * 128), &tm_q, kb * 64, coord(1), coord(2), coord(3), q_full);
  };
  if (warp == C::K_WARP && lane == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
    }
    for (int g = 0; g < NG; ++g) mbar_init(&o_full[g], 1);
    mbar_init(o_final, 1);
    mbar_init(q_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tc::prefetch_tmap(&tm_k);
    tc::prefetch_tmap(&tm_v);
    if (p.q_tma) {
      tc::prefetch_tmap(&tm_q);
      if (q_first) issue_q();
    }
  }

  const int64_t L = p.seq_lens[b];
  const int64_t past = L - (int64_t)p.cur_lens[b];
  const int64_t cap = (int64_t)p.max_pages * BS;
  int64_t kend;
  int ntiles_all, nsplit;
  prefill_tile_range(p, b, t0, C::BM, C::BN, BS, &kend, &ntiles_all, &nsplit);
  if (split >= nsplit) return;  // this query tile needs fewer splits (uniform across the CTA)
  const int j1 = (j0 + p.kt_per_split < ntiles_all) ? j0 + p.kt_per_split : ntiles_all;
  const int ntiles = j1 > j0 ? j1 - j0 : 0;  // tiles of this CTA; tile index = j0 + local

  if (warp == C::K_WARP || warp == C::V_WARP) {
    // ----------------------------------------------------------- producers
    const bool is_k = warp == C::K_WARP;
    if (is_k) {
      if (lane == 0) {
        if (L > cap) set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
        if (p.q_tma && !q_first) issue_q();
      }
      __syncwarp();
      named_bar_arrive(1, C::THREADS);
    } else {
      named_bar_sync(1, C::THREADS);  // barriers initialised
    }
    if (p.early) pdl_wait();  // the append kernel's rows are in the pages about to be copied
    unsigned char* ring = is_k ? sK : sV;
    const CUtensorMap* tmap = is_k ? &tm_k : &tm_v;
    uint64_t* full = is_k ? k_full : v_full;
    uint64_t* empty = is_k ? k_empty : v_empty;
    // Block ids in registers, 32 pages at a time (lane i: page chunk*32+i).
    int chunk = 0;
    int blk_lane = prefill_checked_block(p, blk_pre, pg0 + lane, kend, BS);
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % C::STAGES;
      const uint32_t ph = (uint32_t)(j / C::STAGES) & 1u;
      const int lp = j * C::PAGES;  // first local page of the tile
      if ((lp >> 5) != chunk) {
        chunk = lp >> 5;
        const int64_t page = pg0 + chunk * 32 + lane;
        const int raw = page < p.max_pages ? pt_row[page] : -1;
        blk_lane = prefill_checked_block(p, raw, page, kend, BS);
      }
      if (!warp_wait(&empty[st], ph ^ 1u, p.status, abort_flag)) break;
      // lane pg < PAGES issues the loads of page pg of the tile
      const int my_blk = __shfl_sync(kFullMask, blk_lane, (lp + (lane % C::PAGES)) & 31);
      uint32_t bytes = 0;
#pragma unroll
      for (int pg = 0; pg < C::PAGES; ++pg) {
        const int blk = __shfl_sync(kFullMask, blk_lane, (lp + pg) & 31);
        if (blk >= 0) {
          bytes += (uint32_t)(C::NOP * BS * D * 2);
        } else {
          // Pages that are not loaded must not hold stale or uninitialised
          // bytes: their softmax weight is 0, but 0 * NaN is NaN in P.V.
#pragma unroll
          for (int op = 0; op < C::NOP; ++op)
#pragma unroll
            for (int kb = 0; kb < C::KB; ++kb) {
              const int off = st * C::KV_BYTES + op * C::KV_TILE + kb * (C::BN * 128) + pg * (BS * 128);
              for (int i = lane; i < BS * 8; i += 32) reinterpret_cast<uint4*>(ring + off)[i] = make_uint4(0, 0, 0, 0);
            }
        }
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      // The stage's byte count goes in before any of its loads is issued.
      if (lane == 0) mbar_arrive_expect_tx(&full[st], bytes);
      __syncwarp();
      if (lane < C::PAGES && my_blk >= 0) {
        const int pg = lane;
        const int row = (my_blk * p.H + h) * BS;
        // split variant: the workspace rows hold hi in columns [0, D) and
        // lo in [D, 2D)
#pragma unroll
        for (int op = 0; op < C::NOP; ++op)
#pragma unroll
          for (int kb = 0; kb < C::KB; ++kb) {
            const int off = st * C::KV_BYTES + op * C::KV_TILE + kb * (C::BN * 128) + pg * (BS * 128);
            tc::tma_load_2d(ring + off, tmap, op * D + kb * 64, row, &full[st]);
          }
      }
      __syncwarp();
    }
  } else if (warp == C::QK_WARP || warp == C::PV_WARP) {
    // ------------------------------------------------------- MMA issuers
    // Two issuers, one elected lane each (tcgen05.mma and commit are
    // single-thread instructions): the QK warp issues S(j) = Q.K^T(j) into
    // S buffer j % NSLOT once K(j) has landed and the softmax has read
    // S(j - NSLOT); the PV warp issues O_g += P(j).V(j) for g = j % NG once
    // P(j) and V(j) are ready, and frees P buffer j % NSLOT when done.
    // Operations of different issuers are not ordered with each other, so
    // every hand-over goes through an mbarrier.
    const bool is_qk = warp == C::QK_WARP;
    if (is_qk) {
      tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
      tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    named_bar_sync(1, C::THREADS);
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    constexpr int FMT = !SPLIT && ElemTraits<T>::kDtype == B2PA_DTYPE_BF16 ? 1 : 0;
    constexpr uint32_t idesc_s = tc::idesc_f16(128, C::BN, FMT, 0, 0);
    constexpr uint32_t idesc_o = tc::idesc_f16(128, D, FMT, 0, 1);
    // Descriptors of the operand bases; an operand at byte offset `off` from
    // its base is base + off / 16 (the start-address field, which cannot
    // carry: shared addresses stay below 2^18).
    const uint64_t dQ = tc::smem_desc(smem_u32(sQ), 16, 1024);
    const uint64_t dK = tc::smem_desc(smem_u32(sK), 16, 1024);
    const uint64_t dV = tc::smem_desc(smem_u32(sV), C::BN * 128, 1024);
    const uint64_t dP = tc::smem_desc(smem_u32(sP), 16, 1024);
    if (lane == 0 && is_qk) {
      // Q by TMA: wait for it even without tiles, so that no copy is still
      // landing when the CTA exits.
      const bool q_ok = !p.q_tma || lane_wait(q_full, 0u, p.status, abort_flag);
      for (int j = 0; q_ok && j < ntiles; ++j) {
        const int st = j % C::STAGES, slot = j % NSLOT;
        if (!lane_wait(&k_full[st], (uint32_t)(j / C::STAGES) & 1u, p.status, abort_flag)) break;
        if (j >= NSLOT && !lane_wait(&p_full[slot], (uint32_t)(j / NSLOT - 1) & 1u, p.status, abort_flag)) break;
        tc::fence_after_sync();
        const uint32_t tS = tmem + (uint32_t)slot * C::BN;
        const uint64_t dKs = dK + (uint64_t)((st * C::KV_BYTES) >> 4);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int kb = k >> 2, kk = k & 3;
          const uint64_t a = dQ + (uint64_t)((kb * (C::BM * 128) + kk * 32) >> 4);
          const uint64_t bd = dKs + (uint64_t)((kb * (C::BN * 128) + kk * 32) >> 4);
          tc::mma_f16_ss(tS, a, bd, idesc_s, k > 0);
          if constexpr (SPLIT) {
            tc::mma_f16_ss(tS, a, bd + (uint64_t)(C::KV_TILE >> 4), idesc_s, true);  // q_hi . k_lo
            tc::mma_f16_ss(tS, a + (uint64_t)(C::Q_TILE >> 4), bd, idesc_s, true);   // q_lo . k_hi
          }
        }
        tc::commit(&s_full[slot]);
        tc::commit(&k_empty[st]);
      }
    } else if (lane == 0) {
      bool ok = true;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % C::STAGES, slot = j % NSLOT, g = j % NG;
        if (!lane_wait(&p_full[slot], (uint32_t)(j / NSLOT) & 1u, p.status, abort_flag) ||
            !lane_wait(&v_full[st], (uint32_t)(j / C::STAGES) & 1u, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint64_t dPs = dP + (uint64_t)((slot * C::P_BYTES) >> 4);
        const uint64_t dVs = dV + (uint64_t)((st * C::KV_BYTES) >> 4);
        const uint32_t tO = tmem + (uint32_t)(NSLOT * C::BN + g * D);
#pragma unroll
        for (int k = 0; k < C::BN / 16; ++k) {
          tc::mma_f16_ss(tO, dPs + (uint64_t)(k * 2), dVs + (uint64_t)(k * 128), idesc_o, j >= NG || k > 0);
          if constexpr (SPLIT) {
            tc::mma_f16_ss(tO, dPs + (uint64_t)(k * 2), dVs + (uint64_t)((C::KV_TILE >> 4) + k * 128), idesc_o,
                           true);  // p_hi . v_lo
            tc::mma_f16_ss(tO, dPs + (uint64_t)((C::P_TILE >> 4) + k * 2), dVs + (uint64_t)(k * 128), idesc_o,
                           true);  // p_lo . v_hi
          }
        }
        tc::commit(&o_full[g]);
        tc::commit(&v_empty[st]);
        tc::commit(&p_free[slot]);
      }
      // The epilogue cannot wait on o_full by parity (it may lag by two
      // phases); a separate single-phase barrier marks "all P.V done".
      if (ok && ntiles > 0) tc::commit(o_final);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int g = warp >> 2;     // softmax group
    const int r = tid & 127;     // query row (TMEM lane) of this thread
    const int t = t0 + r;
    // Q: by TMA (issued at kernel entry), by these threads here (16-bit q
    // the tensor map does not take), or already split at kernel entry (fp32).
    if (!SPLIT && !p.q_tma) load_q_threads();
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    named_bar_sync(1, C::THREADS);
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tO = tmem + (uint32_t)(NSLOT * C::BN);  // O of group gg at tO + gg * D
    // Block ids of the CTA's pages (for the visibility mask), validated once.
    {
      const int npg = ntiles * C::PAGES;
      for (int i = tid; i < npg; i += C::SOFTMAX_THREADS) {
        const int64_t page = pg0 + i;
        const int raw = i == tid ? blk_pre : (page < p.max_pages ? pt_row[page] : -1);
        sblk[i] = prefill_checked_block(p, raw, page, kend, BS);
      }
    }
    named_bar_sync(2, C::SOFTMAX_THREADS);
    int64_t row_end = L < past + t + 1 ? L : past + t + 1;
    if (row_end > cap) row_end = cap;
    const uint32_t trow = (uint32_t)((warp & 3) * 32) << 16;
    // O accumulates in TMEM at the scale 2^m_ref.  m_ref only moves when a
    // tile's row max exceeds it by more than kRescale (log2 units), so the
    // P values stay below 2^kRescale and the rescale of O (TMEM load, scale,
    // store) is rare.  Rescaling at the group's i-th tile j waits for the
    // group's previous P.V (tile j - NG): o_full[g] completes one phase per
    // P.V of the group; the p_free wait before it makes P.V(j - NSLOT) done
    // (NSLOT is 2*NG, or NG for the fp32 variant: then that is the group's
    // previous P.V itself), and P.V(j) cannot start before this warp releases
    // P(j), so o_full[g] has completed i-1 or i phases and the parity wait
    // is exact.
    constexpr float kRescale = 8.f;
    // Row maxima are taken on unscaled scores and scaled once (sc > 0); a
    // scale that is not positive is applied to the scores first instead.
    const bool pre_scale = !(p.scale_log2 > 0.f);
    const float sc = pre_scale ? 1.f : p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = g; j < ntiles; j += NG) {
      const int i = j / NG;
      const int slot = j % NSLOT;
      if (!warp_wait(&s_full[slot], (uint32_t)(j / NSLOT) & 1u, p.status, abort_flag)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      float s[64];
      const uint32_t tS = tmem + (uint32_t)slot * C::BN + trow;
      {
        float a[32], c[32];
        tc::tmem_ld32(tS, a);
        tc::tmem_ld32(tS + 32, c);
        tc::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          s[e] = a[e];
          s[32 + e] = c[e];
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
      // Scores stay unscaled (the scale enters the exponent's fma below)
      // unless it is not positive; invisible keys become -inf.
      if (pre_scale) {
#pragma unroll
        for (int e = 0; e < 64; ++e) s[e] *= p.scale_log2;
      }
      if (lim < C::BN || !all_pages) {
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          const bool vis = e < lim && page_ok[e / BS];
          s[e] = vis ? s[e] : -INFINITY;
        }
      }
      // Row max as a tree of three-input maxima (short dependency chains,
      // 36 instructions for 64 values).
      float mx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        mx[e] = fmax3(fmax3(s[e], s[e + 8], s[e + 16]), fmax3(s[e + 24], s[e + 32], s[e + 40]),
                      fmaxf(s[e + 48], s[e + 56]));
      const float mt = sc * fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
      // A row moves its reference max when the tile's max exceeds it by more
      // than kRescale.  Rows that already hold O at the old scale need O and
      // l multiplied by 2^(m_old - m_new); a row with no visible key so far
      // (m = -inf) holds zeros and just adopts the new max.  TMEM accesses
      // and the barrier wait are warp-collective, so the whole warp takes
      // the branch if any lane needs it (other lanes scale by 1).
      // P buffer `slot` is free once P.V(j - NSLOT) is done.  That also makes
      // the group's P.V two tiles back complete, which the rescale's parity
      // wait below relies on.
      if (j >= NSLOT && !warp_wait(&p_free[slot], (uint32_t)(j / NSLOT - 1) & 1u, p.status, abort_flag)) {
        ok = false;
        break;
      }
      const bool need = mt > m + kRescale;
      const float m_new = need ? mt : m;
      const bool scale_o = need && m != -INFINITY;
      const float alpha = scale_o ? fast_exp2(m - m_new) : 1.f;
      m = m_new;
      // P = 2^(s * sc - m), two lanes per fma; a row with no visible key so
      // far (m = -inf) has every s at -inf, so any finite offset gives 0.
      // P is written before the (rare) rescale of O below, which frees the
      // score registers first; P.V cannot start before p_full, after both.
      const float2 sc2 = make_float2(sc, sc);
      const float2 nm2 = make_float2(m == -INFINITY ? 0.f : -m, m == -INFINITY ? 0.f : -m);
      float2 ls[4];  // 8 independent partial sums
#pragma unroll
      for (int e = 0; e < 4; ++e) ls[e] = make_float2(0.f, 0.f);
      unsigned char* sPj = sP + slot * C::P_BYTES;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 x = fma2(make_float2(s[c8 * 8 + 2 * e], s[c8 * 8 + 2 * e + 1]), sc2, nm2);
          pv[2 * e] = fast_exp2(x.x);
          pv[2 * e + 1] = fast_exp2(x.y);
          ls[e] = add2(ls[e], make_float2(pv[2 * e], pv[2 * e + 1]));
        }
        if constexpr (SPLIT) {
          uint4 hi, lo;
          split_f16x8(pv, hi, lo);
          *reinterpret_cast<uint4*>(sPj + tc::sw128_offset(r, c8)) = hi;
          *reinterpret_cast<uint4*>(sPj + C::P_TILE + tc::sw128_offset(r, c8)) = lo;
        } else {
          Vec<T, 8> w;
          w.from_float(pv);
          *reinterpret_cast<uint4*>(sPj + tc::sw128_offset(r, c8)) = w.w;
        }
      }
      const float2 l01 = add2(ls[0], ls[1]), l23 = add2(ls[2], ls[3]);
      const float tile_sum = (l01.x + l01.y) + (l23.x + l23.y);
      if (i > 0 && __any_sync(kFullMask, scale_o)) {
        // wait for the group's previous P.V before touching its O
        if (!warp_wait(&o_full[g], (uint32_t)(i - 1) & 1u, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int cb = 0; cb < D / 32; ++cb) {
          float ov[32];
          tc::tmem_ld32(tO + g * D + trow + cb * 32, ov);
          tc::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] *= alpha;
          tc::tmem_st32(tO + g * D + trow + cb * 32, ov);
        }
        tc::tmem_wait_st();
        l *= alpha;
      }
      l += tile_sum;
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[slot]);
    }
    // ---------------------------------------------------------- epilogue
    // Merge the groups' (m, l, O) for this row: weights 2^(m_g - M).  Group g
    // writes columns [g*D/NG, (g+1)*D/NG) of the row.
    float M = m, wgt[NG];
    wgt[0] = 1.f;
    float lsum = l;
    if constexpr (NG > 1) {
      sML[(g * C::BM + r) * 2] = m;
      sML[(g * C::BM + r) * 2 + 1] = l;
      named_bar_sync(2, C::SOFTMAX_THREADS);
      float mg[NG], lg[NG];
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) {
        mg[gg] = sML[(gg * C::BM + r) * 2];
        lg[gg] = sML[(gg * C::BM + r) * 2 + 1];
      }
      M = mg[0];
#pragma unroll
      for (int gg = 1; gg < NG; ++gg) M = fmaxf(M, mg[gg]);
      lsum = 0.f;
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) {
        wgt[gg] = mg[gg] == -INFINITY ? 0.f : fast_exp2(mg[gg] - M);
        lsum = fmaf(lg[gg], wgt[gg], lsum);
      }
    }
    constexpr int DC = D / NG;  // columns this thread writes
    const int c0 = g * DC;
    const bool have_o = ok && ntiles > 0 && warp_wait(o_final, 0u, p.status, abort_flag);  // warp-uniform
    if (have_o) tc::fence_after_sync();
    const bool partial = nsplit > 1;
    const float inv = 1.f / fmaxf(lsum, 1e-9f);
    const int64_t pslot = (((int64_t)b * p.H + h) * p.T + t) * p.nsplit_max + split;
    // 32 columns at a time (TMEM loads are warp-collective: every lane runs them)
#pragma unroll
    for (int cb = 0; cb < DC / 32; ++cb) {
      float o[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) o[e] = 0.f;
      if (have_o) {
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) {
          if (gg >= ntiles) break;  // group without tiles: its O was never written
          float ov[32];
          tc::tmem_ld32(tO + gg * D + trow + c0 + cb * 32, ov);
          tc::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = NG > 1 ? fmaf(wgt[gg], ov[e], o[e]) : ov[e];
        }
      }
      if (t >= p.T) continue;
      if (partial) {
        float4* po = reinterpret_cast<float4*>(p.part_o + pslot * D + c0 + cb * 32);
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) po[c4] = make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]);
      } else {
        T* orow = static_cast<T*>(p.out) + (int64_t)b * p.so_b + (int64_t)h * p.so_h + (int64_t)t * p.so_t + c0 +
                  cb * 32;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = o[c8 * 8 + e] * inv;
          if constexpr (SPLIT) {
            float4* o4 = reinterpret_cast<float4*>(orow + c8 * 8);
            o4[0] = make_float4(f[0], f[1], f[2], f[3]);
            o4[1] = make_float4(f[4], f[5], f[6], f[7]);
          } else {
            Vec<T, 8> w;
            w.from_float(f);
            *reinterpret_cast<uint4*>(orow + c8 * 8) = w.w;
          }
        }
      }
    }
    tc::fence_before_sync();
    if (t < p.T && partial && g == 0) {
      p.part_ml[2 * pslot] = M;
      p.part_ml[2 * pslot + 1] = lsum;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == C::QK_WARP) {
    tc::fence_after_sync();
    tc::tmem_dealloc(*tmem_slot, C::TMEM_COLS);
  }
}

// One warp per (sequence, head, query row) whose query tile was split:
// log-sum-exp merge of the split partials, then the reference's normalisation.
// Serves both prefill kernels (p.bm gives their query-tile height).
template <typename T, int D, int BS>
__global__ void __launch_bounds__(256) prefill_combine_kernel(PfTcParams p) {
  // launched as a programmatic dependent of the kernel that wrote the partials
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= (int64_t)p.B * p.H * p.T) return;
  const int t = (int)(row % p.T);
  const int h = (int)((row / p.T) % p.H);
  const int b = (int)(row / ((int64_t)p.T * p.H));
  int64_t kend;
  int ntiles, nsplit;
  prefill_tile_range(p, b, (t / p.bm) * p.bm, p.bm, 64, BS, &kend, &ntiles, &nsplit);
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

// The fp32 variant's first step: copies every page that the prefill of
// sequence b reads (pages holding keys below min(seq_len, table width)) of K
// and of V into the workspace as fp16 hi/lo rows -- row (slot * H + h) * BS
// + r holds hi in columns [0, D) and lo in [D, 2D), slot = b * max_pages +
// page -- and writes the slot table the kernel walks in place of the block
// table: -1 for a page it must not read (past the sequence, a negative
// entry, or a block id outside the pool, which is also reported).
struct PfSplitArgs {
  float* k_pool;  // written only by the fused append (rows of k_new / v_new)
  float* v_pool;
  const int32_t* page_table;
  int64_t pt_stride;
  int max_pages;
  const int32_t* seq_lens;
  int64_t num_blocks;
  int H;
  __half* k_split;
  __half* v_split;
  int32_t* slots;
  uint32_t* range_flag;
  uint32_t epoch;
  int32_t* status;
  // Fused KV append (b2pa_paged_prefill_append; app_len null: none): rows
  // t < min(app_len[b], T) of k_new / v_new go to positions app_start[b] + t,
  // which must end at seq_lens[b].  The page copy takes those rows from
  // k_new / v_new and also writes them into the pool.  seq_out (optional)
  // receives seq_lens as int64.
  const float* k_new;
  const float* v_new;
  int64_t skn[3], svn[3];
  const int32_t* app_start;
  const int32_t* app_len;
  int T;
  int64_t* seq_out;
};

template <int D, int BS>
__global__ void __launch_bounds__(128) prefill_split_pages_kernel(PfSplitArgs a) {
  pdl_launch_dependents();  // the tensor-core kernel may launch now; it waits for this grid
  const int i = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  int64_t kend = a.seq_lens[b];
  const int64_t cap = (int64_t)a.max_pages * BS;
  kend = kend < cap ? kend : cap;
  const int64_t slot = (int64_t)b * a.max_pages + i;
  int64_t blk = -1;
  if ((int64_t)i * BS < kend) {
    const int32_t raw = a.page_table[(int64_t)b * a.pt_stride + i];
    if (raw >= 0 && raw < a.num_blocks) {
      blk = raw;
    } else if (raw >= a.num_blocks && h == 0 && threadIdx.x == 0) {
      set_status(a.status, B2PA_ERR_BAD_BLOCK_ID);
    }
  }
  if (h == 0 && threadIdx.x == 0) a.slots[slot] = (int32_t)(blk >= 0 ? slot : -1);
  // positions [app_lo, app_hi) of sequence b come from k_new / v_new
  int64_t app_lo = 0, app_hi = 0;
  if (a.app_len != nullptr) {
    int len = a.app_len[b];
    len = len < a.T ? len : a.T;
    if (len > 0) {
      app_lo = a.app_start[b];
      app_hi = app_lo + len;
      if (app_lo < 0 || app_hi != (int64_t)a.seq_lens[b]) {  // not the chunk that ends the sequence
        if (i == 0 && h == 0 && threadIdx.x == 0) set_status(a.status, B2PA_ERR_INVALID_ARGUMENT);
        app_lo = app_hi = 0;
      }
    }
    if (a.seq_out != nullptr && i == 0 && h == 0 && threadIdx.x == 0) a.seq_out[b] = a.seq_lens[b];
  }
  if (blk < 0) return;
  const int64_t src = ((blk * a.H + h) * BS) * D;
  const int64_t dst = ((slot * a.H + h) * BS) * (2 * D);
  bool in_range = true;
  for (int idx = threadIdx.x; idx < BS * D / 8; idx += blockDim.x) {
    const int r = idx / (D / 8), c8 = idx - (idx / (D / 8)) * (D / 8);
    const int64_t pos = (int64_t)i * BS + r;
    const bool fresh = pos >= app_lo && pos < app_hi;
    // Both rows (K and V) are loaded before anything is stored, so the four
    // 16-byte loads are in flight together (the stores below could alias
    // them as far as the compiler knows).
    float4 x[2][2];
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const float4* s4;
      if (fresh) {
        const int64_t t = pos - app_lo;
        const int64_t* sn = kv ? a.svn : a.skn;
        s4 = reinterpret_cast<const float4*>((kv ? a.v_new : a.k_new) + (int64_t)b * sn[0] + (int64_t)h * sn[1] +
                                             t * sn[2] + c8 * 8);
      } else {
        s4 = reinterpret_cast<const float4*>((kv ? a.v_pool : a.k_pool) + src + (int64_t)r * D + c8 * 8);
      }
      x[kv][0] = s4[0];
      x[kv][1] = s4[1];
    }
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const float4 x0 = x[kv][0], x1 = x[kv][1];
      if (fresh) {
        float* pool_row = (kv ? a.v_pool : a.k_pool) + src + (int64_t)r * D + c8 * 8;
        reinterpret_cast<float4*>(pool_row)[0] = x0;
        reinterpret_cast<float4*>(pool_row)[1] = x1;
      }
      const float f[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) in_range = in_range && fabsf(f[e]) < kSplitRange;
      uint4 hi, lo;
      split_f16x8(f, hi, lo);
      __half* d = (kv ? a.v_split : a.k_split) + dst + (int64_t)r * (2 * D) + c8 * 8;
      *reinterpret_cast<uint4*>(d) = hi;
      *reinterpret_cast<uint4*>(d + D) = lo;
    }
  }
  if (!in_range) *a.range_flag = a.epoch;
}

// ----------------------------------------------------------------- host ---
bool encode_pool_tensor_map(CUtensorMap* map, const void* pool, int64_t rows, int D, int block_size, int dtype);
bool encode_q_tensor_map(CUtensorMap* map, const void* q, int B, int H, int T, int D, const int64_t sq[3], int dtype,
                         int dim_of[3]);

// epoch: the fp32 variant's number of this call (marks the range flag).
template <typename T, int D, int BS>
int launch_prefill_tc(const AttnArgs& a, cudaStream_t stream, uint32_t epoch = 0) {
  constexpr bool SPLIT = kPfSplit<T>;
  using C = PfTcCfg<D, BS, SPLIT>;
  const PrefillPlan plan = make_prefill_plan(a.B, a.H, a.T, a.D, a.max_pages, BS, a.dtype);
  if (plan.bytes > 0 && (!a.workspace || a.workspace_bytes < plan.bytes))
    return set_error(B2PA_ERR_WORKSPACE, "paged_prefill: workspace of %zu bytes, %zu needed", a.workspace_bytes,
                     plan.bytes);
  CUtensorMap tmk, tmv;
  uint32_t* range_flag = nullptr;
  const int32_t* table = a.page_table;
  int64_t pt_stride = a.pt_stride;
  int64_t num_blocks = a.num_blocks;
  if constexpr (SPLIT) {
    if (!plan.split_tc) return set_error(B2PA_ERR_UNSUPPORTED, "paged_prefill: fp32 split plan not applicable");
    char* ws = static_cast<char*>(a.workspace);
    PfSplitArgs sa;
    sa.k_pool = const_cast<float*>(static_cast<const float*>(a.k_pool));
    sa.v_pool = const_cast<float*>(static_cast<const float*>(a.v_pool));
    sa.k_new = static_cast<const float*>(a.k_new);
    sa.v_new = static_cast<const float*>(a.v_new);
    for (int i = 0; i < 3; ++i) {
      sa.skn[i] = a.skn[i];
      sa.svn[i] = a.svn[i];
    }
    sa.app_start = a.app_start;
    sa.app_len = a.app_len;
    sa.T = a.T;
    sa.seq_out = a.seq_out;
    sa.page_table = a.page_table;
    sa.pt_stride = a.pt_stride;
    sa.max_pages = a.max_pages;
    sa.seq_lens = a.seq_lens;
    sa.num_blocks = a.num_blocks;
    sa.H = a.H;
    sa.k_split = reinterpret_cast<__half*>(ws + plan.off_split_k);
    sa.v_split = reinterpret_cast<__half*>(ws + plan.off_split_v);
    sa.slots = reinterpret_cast<int32_t*>(ws + plan.off_slots);
    sa.range_flag = reinterpret_cast<uint32_t*>(ws + plan.off_flag);
    sa.epoch = epoch;
    sa.status = a.status;
    range_flag = sa.range_flag;
    const int64_t nslots = (int64_t)a.B * a.max_pages;
    const int64_t rows = nslots * a.H * BS;
    if (!encode_pool_tensor_map(&tmk, sa.k_split, rows, 2 * D, BS, B2PA_DTYPE_F16) ||
        !encode_pool_tensor_map(&tmv, sa.v_split, rows, 2 * D, BS, B2PA_DTYPE_F16))
      return set_error(B2PA_ERR_CUDA, "paged_prefill: cuTensorMapEncodeTiled failed for the split pages");
    prefill_split_pages_kernel<D, BS><<<dim3((unsigned)a.max_pages, (unsigned)a.H, (unsigned)a.B), 128, 0, stream>>>(
        sa);
    table = sa.slots;
    pt_stride = a.max_pages;
    num_blocks = nslots;
  } else {
    const int64_t rows = a.num_blocks * a.H * BS;
    if (!encode_pool_tensor_map(&tmk, a.k_pool, rows, D, BS, a.dtype) ||
        !encode_pool_tensor_map(&tmv, a.v_pool, rows, D, BS, a.dtype))
      return set_error(B2PA_ERR_CUDA, "paged_prefill: cuTensorMapEncodeTiled failed for the pools");
  }
  PfTcParams p;
  p.q = a.q;
  p.sq_b = a.sq[0];
  p.sq_h = a.sq[1];
  p.sq_t = a.sq[2];
  p.page_table = table;
  p.pt_stride = pt_stride;
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
  p.num_blocks = num_blocks;
  p.scale_log2 = a.scale * kLog2e;
  p.status = a.status;
  p.kt_per_split = plan.kt_per_split;
  p.nsplit_max = plan.nsplit_max;
  p.bm = C::BM;
  p.part_o = nullptr;
  p.part_ml = nullptr;
  p.range_flag = range_flag;
  p.epoch = epoch;
  p.early = (!SPLIT && a.after_append) ? 1 : 0;
  if (plan.nsplit_max > 1) {
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
  // 16-bit q: a tensor map for its TMA load (q layouts the driver refuses
  // are loaded by the softmax threads).
  CUtensorMap tmq = tmk;
  p.q_tma = 0;
  p.q_dim[0] = 1;
  p.q_dim[1] = 2;
  p.q_dim[2] = 3;
  if (!SPLIT) {
    const int64_t sq[3] = {a.sq[0], a.sq[1], a.sq[2]};
    p.q_tma = encode_q_tensor_map(&tmq, a.q, a.B, a.H, a.T, a.D, sq, a.dtype, p.q_dim) ? 1 : 0;
    if (!p.q_tma) tmq = tmk;  // not read
  }
  e = launch_pdl(kern, grid, dim3(C::THREADS), smem, stream, tmk, tmv, tmq, p);
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_prefill_tc launch: %s", cudaGetErrorString(e));
  if (plan.nsplit_max > 1) {
    const int64_t rows = (int64_t)a.B * a.H * a.T;
    e = launch_pdl(prefill_combine_kernel<T, D, BS>, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, stream, p);
    if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "prefill_combine launch: %s", cudaGetErrorString(e));
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_prefill_tc launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

}  // namespace b2pa
