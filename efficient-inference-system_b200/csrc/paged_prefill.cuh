// paged_prefill.cuh -- chunked-prefill paged attention, fp32 CUDA-core path.
//
// Replaces the Triton prefill kernel of the reference
// (src/kernels/triton_paged_attention.py:88-176, launcher :220-258), which
// runs one program per (sequence, head, query row) and re-reads every key it
// sees for each row.  Semantics (src/kernels/reference_paged_attention.py:
// 31-57): query row t of sequence b sits at absolute position
// pos = seq_len - cur_len + t and sees keys 0 .. min(seq_len, pos + 1) - 1;
// rows past cur_len (padding) therefore see the whole sequence; a row with
// no visible key is zero.
//
// This path computes in fp32 FMA for every element type: one CTA per
// (32-row query tile, head, sequence), key tiles of 64 tokens gathered
// page by page through the block table into shared memory, and an online
// softmax in the log2 domain.  Each key is read once per query tile instead
// of once per query row.
#pragma once

#include <algorithm>
#include <climits>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace b2pa {

__device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

constexpr int kPfTQ = 32;   // query rows per CTA
constexpr int kPfTK = 64;   // keys per tile
constexpr int kPfThreads = 256;

struct PrefillParams {
  const void* q;
  int64_t sq_b, sq_h, sq_t;
  const void* k_pool;
  const void* v_pool;
  int64_t num_blocks;
  const int32_t* page_table;
  int64_t pt_stride;
  int max_pages;
  const int32_t* seq_lens;
  const int32_t* cur_lens;
  void* out;
  int64_t so_b, so_h, so_t;
  int B, H, T;
  float qscale;
  int32_t* status;
  // Key-range split (fp32 tiled kernel only): CTA x = query_tile * nsplit_max
  // + s covers key tiles [s*kt_per_split, (s+1)*kt_per_split); split rows
  // write fp32 partials merged by prefill_combine_kernel.
  int kt_per_split;
  int nsplit_max;
  float* part_o;   // [B, H, T, nsplit_max, D]
  float* part_ml;  // [B, H, T, nsplit_max, 2]
  // Backup launch (general kernel only): when not null, the kernel does
  // nothing unless *run_if == run_epoch.
  const uint32_t* run_if;
  uint32_t run_epoch;
};

template <int D>
struct PrefillSmem {
  static constexpr int QLD = D + 1;   // padded row pitch (floats)
  static constexpr int KLD = D + 1;
  static constexpr int VLD = D;
  static constexpr int PLD = kPfTK + 1;
  static constexpr int Q_FLOATS = kPfTQ * QLD;
  static constexpr int K_FLOATS = kPfTK * KLD;
  static constexpr int V_FLOATS = kPfTK * VLD;
  static constexpr int P_FLOATS = kPfTQ * PLD;
  static constexpr size_t BYTES = 4ull * (Q_FLOATS + K_FLOATS + V_FLOATS + P_FLOATS + kPfTK);
};

// One (32 query rows, head, sequence) tile of the general kernel.
template <typename T, int D, int BS>
__device__ __forceinline__ void paged_prefill_simt_tile(const PrefillParams& p, int tile, int h, int b, float* psm) {
  using S = PrefillSmem<D>;
  float* Qs = psm;
  float* Ks = Qs + S::Q_FLOATS;
  float* Vs = Ks + S::K_FLOATS;
  float* Ps = Vs + S::V_FLOATS;
  int* Kok = reinterpret_cast<int*>(Ps + S::P_FLOATS);  // key row came from a real page

  const int t0 = tile * kPfTQ;
  const int tid = threadIdx.x;
  if (t0 >= p.T) return;

  const int64_t L = p.seq_lens[b];
  const int64_t past = L - (int64_t)p.cur_lens[b];
  const T* qg = static_cast<const T*>(p.q);
  for (int i = tid; i < kPfTQ * D; i += kPfThreads) {
    const int r = i / D, d = i - (i / D) * D;
    const int t = t0 + r;
    Qs[r * S::QLD + d] = t < p.T ? to_f32(qg[(int64_t)b * p.sq_b + (int64_t)h * p.sq_h + (int64_t)t * p.sq_t + d]) * p.qscale : 0.f;
  }

  const int t_last = (t0 + kPfTQ < p.T ? t0 + kPfTQ : p.T) - 1;
  const int64_t cap = (int64_t)p.max_pages * BS;
  if (L > cap && tid == 0) set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
  int64_t kend = min64(L, past + t_last + 1);
  kend = min64(kend, cap);
  if (kend < 0) kend = 0;

  const int row = tid >> 3;  // 32 rows x 8 threads
  const int sub = tid & 7;
  const int t = t0 + row;
  int64_t row_end = min64(L, past + t + 1);
  row_end = min64(row_end, cap);

  constexpr int OD = D / 8;  // output columns per thread (sub + 8*i)
  float o[OD];
#pragma unroll
  for (int i = 0; i < OD; ++i) o[i] = 0.f;
  float m = -INFINITY, l_part = 0.f;

  const T* kp = static_cast<const T*>(p.k_pool);
  const T* vp = static_cast<const T*>(p.v_pool);
  constexpr int CHV = (16 / (int)sizeof(T)) < D ? (16 / (int)sizeof(T)) : D;  // elements per vector load
  constexpr int VPR = D / CHV;                                               // vector loads per row
  using VL = Vec<T, CHV>;

  for (int64_t k0 = 0; k0 < kend; k0 += kPfTK) {
    __syncthreads();
    for (int i = tid; i < kPfTK * VPR; i += kPfThreads) {
      const int r = i / VPR, cc = i - (i / VPR) * VPR;
      const int64_t tok = k0 + r;
      float kf[CHV], vf[CHV];
      bool have = false;
      if (tok < kend) {
        const int32_t blk = p.page_table[(int64_t)b * p.pt_stride + tok / BS];
        if (blk >= 0 && blk < p.num_blocks) {
          const int64_t off = (((int64_t)blk * p.H + h) * BS + (tok % BS)) * D + cc * CHV;
          VL kv, vv;
          kv.w = ld_global_nc<typename VL::Word>(kp + off);
          vv.w = ld_global_nc<typename VL::Word>(vp + off);
          kv.to_float(kf);
          vv.to_float(vf);
          have = true;
        } else if (blk >= p.num_blocks) {
          set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
        }
      }
      if (cc == 0) Kok[r] = have ? 1 : 0;
#pragma unroll
      for (int e = 0; e < CHV; ++e) {
        Ks[r * S::KLD + cc * CHV + e] = have ? kf[e] : 0.f;
        Vs[r * S::VLD + cc * CHV + e] = have ? vf[e] : 0.f;
      }
    }
    __syncthreads();

    float s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = 0.f;
    const float* qrow = Qs + row * S::QLD;
#pragma unroll 8
    for (int d = 0; d < D; ++d) {
      const float qd = qrow[d];
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] = fmaf(qd, Ks[(sub + 8 * j) * S::KLD + d], s[j]);
    }
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t col = k0 + sub + 8 * j;
      if (col >= row_end || !Kok[sub + 8 * j]) s[j] = -INFINITY;
      mt = fmaxf(mt, s[j]);
    }
    mt = fmaxf(mt, __shfl_xor_sync(kFullMask, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(kFullMask, mt, 2));
    mt = fmaxf(mt, __shfl_xor_sync(kFullMask, mt, 4));
    const float m_new = fmaxf(m, mt);
    const bool live = m_new != -INFINITY;
    const float alpha = live ? exp2f(m - m_new) : 1.f;
    float* prow = Ps + row * S::PLD;
    float lsum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float pj = live ? exp2f(s[j] - m_new) : 0.f;
      prow[sub + 8 * j] = pj;
      lsum += pj;
    }
    l_part = l_part * alpha + lsum;
    m = m_new;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < OD; ++i) o[i] *= alpha;
#pragma unroll 4
    for (int kk = 0; kk < kPfTK; ++kk) {
      const float pk = prow[kk];
      const float* vrow = Vs + kk * S::VLD + sub;
#pragma unroll
      for (int i = 0; i < OD; ++i) o[i] = fmaf(pk, vrow[8 * i], o[i]);
    }
  }

  float l = l_part;
  l += __shfl_xor_sync(kFullMask, l, 1);
  l += __shfl_xor_sync(kFullMask, l, 2);
  l += __shfl_xor_sync(kFullMask, l, 4);
  if (t < p.T) {
    const float den = fmaxf(l, 1e-9f);
    T* og = static_cast<T*>(p.out) + (int64_t)b * p.so_b + (int64_t)h * p.so_h + (int64_t)t * p.so_t;
#pragma unroll
    for (int i = 0; i < OD; ++i) og[sub + 8 * i] = from_f32<T>(o[i] / den);
  }
}

template <typename T, int D, int BS>
__global__ void __launch_bounds__(kPfThreads) paged_prefill_simt_kernel(PrefillParams p) {
  extern __shared__ __align__(16) float psm[];
  if (p.run_if != nullptr) {
    // A backup launch (programmatic): nothing to redo unless the flag says
    // so.  It runs as a persistent grid (one CTA per SM) over the tiles, so
    // that the usual case -- check the flag, exit -- retires few CTAs.
    pdl_wait();
    if (*p.run_if != p.run_epoch) return;
    const int nx = (p.T + kPfTQ - 1) / kPfTQ;
    const int64_t total = (int64_t)nx * p.H * p.B;
    for (int64_t it = blockIdx.x; it < total; it += gridDim.x) {
      __syncthreads();  // the previous tile's threads are done with shared memory
      paged_prefill_simt_tile<T, D, BS>(p, (int)(it % nx), (int)((it / nx) % p.H), (int)(it / ((int64_t)nx * p.H)),
                                        psm);
    }
    return;
  }
  paged_prefill_simt_tile<T, D, BS>(p, blockIdx.x, blockIdx.y, blockIdx.z, psm);
}

// run_if / run_epoch: a backup launch, which does nothing unless *run_if ==
// run_epoch (the fp16-split tensor-core kernel met an input out of range).
template <typename T, int D, int BS>
int launch_prefill_simt(const AttnArgs& a, cudaStream_t stream, const uint32_t* run_if = nullptr,
                        uint32_t run_epoch = 0) {
  PrefillParams p;
  p.q = a.q;
  p.sq_b = a.sq[0];
  p.sq_h = a.sq[1];
  p.sq_t = a.sq[2];
  p.k_pool = a.k_pool;
  p.v_pool = a.v_pool;
  p.num_blocks = a.num_blocks;
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
  p.qscale = a.scale * kLog2e;
  p.status = a.status;
  p.kt_per_split = INT_MAX;  // no key split in this kernel
  p.nsplit_max = 1;
  p.run_if = run_if;
  p.run_epoch = run_epoch;
  p.part_o = nullptr;
  p.part_ml = nullptr;
  const size_t smem = PrefillSmem<D>::BYTES;
  if (smem > (size_t)device_max_smem_optin())
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_prefill: %zu bytes of shared memory exceed the device limit", smem);
  auto kern = paged_prefill_simt_kernel<T, D, BS>;
  int rc_attr = set_max_dynamic_smem_cached(reinterpret_cast<const void*>(kern), (int)smem);
  if (rc_attr != B2PA_OK) return rc_attr;
  cudaError_t e;
  dim3 grid((a.T + kPfTQ - 1) / kPfTQ, a.H, a.B);
  if (run_if != nullptr) {
    const int64_t total = (int64_t)grid.x * grid.y * grid.z;
    const int64_t sms = device_sm_count();
    e = launch_pdl(kern, dim3((unsigned)(total < sms ? total : sms)), dim3(kPfThreads), smem, stream, p);
    if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_prefill launch: %s", cudaGetErrorString(e));
  } else {
    kern<<<grid, kPfThreads, smem, stream>>>(p);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_prefill launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

template <typename T>
int dispatch_prefill(const AttnArgs& a, cudaStream_t s) {
#define B2PA_PF_CASE(DD, BB) \
  if (a.D == DD && a.block_size == BB) return launch_prefill_simt<T, DD, BB>(a, s);
#define B2PA_PF_D(DD) B2PA_PF_CASE(DD, 8) B2PA_PF_CASE(DD, 16) B2PA_PF_CASE(DD, 32)
  B2PA_PF_D(16)
  B2PA_PF_D(32)
  B2PA_PF_D(64)
  B2PA_PF_D(128)
  B2PA_PF_D(256)
#undef B2PA_PF_D
#undef B2PA_PF_CASE
  return set_error(B2PA_ERR_UNSUPPORTED, "paged_prefill: head_dim %d / block_size %d not built", a.D, a.block_size);
}

}  // namespace b2pa
