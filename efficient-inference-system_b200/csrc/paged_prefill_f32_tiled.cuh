// paged_prefill_f32_tiled.cuh -- chunked-prefill paged attention for fp32
// pools with head_dim 64 or 128, on the CUDA cores with register tiling.
//
// Same semantics as paged_prefill_simt_kernel (src/kernels/
// reference_paged_attention.py:31-57; the Triton prefill kernel it replaces
// is src/kernels/triton_paged_attention.py:88-176): query row t of sequence b
// sees keys 0 .. min(seq_len, seq_len - cur_len + t + 1) - 1; a row with no
// visible key is zero.  Exact fp32 FMA throughout, as the fp32 tolerance of
// the path (rtol 1e-4) needs; TF32 tensor cores would not meet it.
//
// One CTA = (64 query rows, head, sequence), 256 threads as a 16 x 16 grid.
// Thread (ty, tx) owns query rows ty + 16a and keys tx + 16b (a, b < 4) of a
// 64-key tile for S = Q.K^T, and rows ty + 16a x head-dim columns
// 4*tx + 64c (float4 each) of O.  Operands are read from shared memory as
// float4 along the contraction dimension, so every 16-byte shared load feeds
// 4 FMAs per owned row or key (8 FMAs per load on average) instead of one.
// K and V tiles of 64 keys are gathered page by page through the block table
// with cp.async (16 bytes per thread, zero-fill for missing keys) into a
// two-stage ring, so the gather of tile j+1 overlaps the math on tile j.
// Long key ranges are split across CTAs (at most 8 key tiles each) whose
// partials the combine kernel merges, so the longest causal rows do not set
// the length of the launch.
// Row pitch D + 4 floats keeps float4 alignment and makes the eight rows
// that one quarter-warp reads fall into distinct bank groups.
#pragma once

#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "paged_prefill.cuh"
#include "paged_prefill_tc.cuh"  // prefill_combine_kernel

namespace b2pa {

template <int D>
struct PfF32Cfg {
  static constexpr int TQ = 64;             // query rows per CTA
  static constexpr int TK = 64;             // keys per tile
  static constexpr int THREADS = 256;
  static constexpr int LD = D + 4;          // row pitch (floats) of Q, K, V
  static constexpr int PLD = TK + 4;        // row pitch of P
  static constexpr int DC = D / 64;         // float4 column groups of O per thread
  static constexpr int Q_FLOATS = TQ * LD;
  static constexpr int KV_FLOATS = TK * LD;
  static constexpr int P_FLOATS = TQ * PLD;
  // Q | K[2] | V[2] | P | key-present flags[2][TK]
  static constexpr size_t BYTES = 4ull * (Q_FLOATS + 4 * KV_FLOATS + P_FLOATS + 2 * TK);
  static_assert(D == 64 || D == 128, "tiled fp32 prefill is built for head_dim 64 and 128");
};

// 16-byte asynchronous global -> shared copy; src_bytes = 0 writes zeros.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int D, int BS>
__global__ void __launch_bounds__(256, D == 64 ? 2 : 1) paged_prefill_f32_tiled_kernel(PrefillParams p) {
  using C = PfF32Cfg<D>;
  extern __shared__ __align__(16) float fsm[];
  float* Qs = fsm;
  float* Ks = Qs + C::Q_FLOATS;          // [2][TK][LD]
  float* Vs = Ks + 2 * C::KV_FLOATS;     // [2][TK][LD]
  float* Ps = Vs + 2 * C::KV_FLOATS;     // [TQ][PLD]
  int* Kok = reinterpret_cast<int*>(Ps + C::P_FLOATS);  // [2][TK]

  const int split = blockIdx.x % p.nsplit_max;
  const int t0 = (blockIdx.x / p.nsplit_max) * C::TQ;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  if (t0 >= p.T) return;

  const int64_t L = p.seq_lens[b];
  const int64_t past = L - (int64_t)p.cur_lens[b];
  const int64_t cap = (int64_t)p.max_pages * BS;
  if (L > cap && tid == 0) set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
  const int t_last = (t0 + C::TQ < p.T ? t0 + C::TQ : p.T) - 1;
  int64_t kend = min64(min64(L, past + t_last + 1), cap);
  if (kend < 0) kend = 0;
  const int ntiles_all = (int)((kend + C::TK - 1) / C::TK);
  int nsplit = (ntiles_all + p.kt_per_split - 1) / p.kt_per_split;
  if (nsplit < 1) nsplit = 1;
  if (split >= nsplit) return;  // uniform across the CTA
  const int j0 = split * p.kt_per_split;
  const int j1 = j0 + p.kt_per_split < ntiles_all ? j0 + p.kt_per_split : ntiles_all;

  const float* kp = static_cast<const float*>(p.k_pool);
  const float* vp = static_cast<const float*>(p.v_pool);
  const int32_t* pt_row = p.page_table + (int64_t)b * p.pt_stride;

  // Gather of key tile j into ring stage st: thread i copies 16-byte chunk
  // (i % (D/4)) of key (i / (D/4)) for K and for V.
  auto issue_tile = [&](int j, int st) {
    constexpr int CPR = D / 4;
    for (int i = tid; i < C::TK * CPR; i += C::THREADS) {
      const int c = i / CPR, ch = i - c * CPR;
      const int64_t tok = (int64_t)j * C::TK + c;
      const float* ks = kp;
      const float* vs = vp;
      int bytes = 0;
      if (tok < kend) {
        const int32_t blk = __ldg(pt_row + tok / BS);
        if (blk >= 0 && blk < p.num_blocks) {
          const int64_t off = (((int64_t)blk * p.H + h) * BS + (tok % BS)) * D + ch * 4;
          ks = kp + off;
          vs = vp + off;
          bytes = 16;
        } else if (blk >= p.num_blocks && ch == 0) {
          set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
        }
      }
      cp_async16(Ks + st * C::KV_FLOATS + c * C::LD + ch * 4, ks, bytes);
      cp_async16(Vs + st * C::KV_FLOATS + c * C::LD + ch * 4, vs, bytes);
      if (ch == 0) Kok[st * C::TK + c] = bytes ? 1 : 0;
    }
    cp_async_commit();
  };

  if (j1 > j0) issue_tile(j0, 0);

  // Q rows, pre-scaled by scale * log2(e); zeros past T.
  const float* qg = static_cast<const float*>(p.q);
  for (int i = tid; i < C::TQ * D; i += C::THREADS) {
    const int r = i / D, d = i - (i / D) * D;
    const int t = t0 + r;
    Qs[r * C::LD + d] =
        t < p.T ? qg[(int64_t)b * p.sq_b + (int64_t)h * p.sq_h + (int64_t)t * p.sq_t + d] * p.qscale : 0.f;
  }

  // Per owned row: visible-key limit, running max, partial denominator.
  int64_t row_end[4];
  float m[4], l_part[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int t = t0 + ty + 16 * a;
    row_end[a] = min64(min64(L, past + t + 1), cap);
    m[a] = -INFINITY;
    l_part[a] = 0.f;
  }
  float4 o[4][C::DC];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int c = 0; c < C::DC; ++c) o[a][c] = make_float4(0.f, 0.f, 0.f, 0.f);

  for (int j = j0; j < j1; ++j) {
    const int st = (j - j0) & 1;
    if (j + 1 < j1) {
      issue_tile(j + 1, st ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // tile j (and Q) visible to every thread

    // S = Q.K^T for rows ty+16a, keys tx+16b.
    const float* Kt = Ks + st * C::KV_FLOATS;
    float s[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) s[a][bb] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; d += 4) {
      float4 qa[4], kb[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) qa[a] = *reinterpret_cast<const float4*>(Qs + (ty + 16 * a) * C::LD + d);
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) kb[bb] = *reinterpret_cast<const float4*>(Kt + (tx + 16 * bb) * C::LD + d);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
          s[a][bb] = fmaf(qa[a].x, kb[bb].x, s[a][bb]);
          s[a][bb] = fmaf(qa[a].y, kb[bb].y, s[a][bb]);
          s[a][bb] = fmaf(qa[a].z, kb[bb].z, s[a][bb]);
          s[a][bb] = fmaf(qa[a].w, kb[bb].w, s[a][bb]);
        }
    }

    // Mask, online softmax per row (the 16 tx threads of a row reduce by
    // shuffles), P to shared memory.
    const int64_t k0 = (int64_t)j * C::TK;
    bool kok[4];
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) kok[bb] = Kok[st * C::TK + tx + 16 * bb] != 0;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      float mt = -INFINITY;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const int64_t key = k0 + tx + 16 * bb;
        if (key >= row_end[a] || !kok[bb]) s[a][bb] = -INFINITY;
        mt = fmaxf(mt, s[a][bb]);
      }
#pragma unroll
      for (int x = 1; x < 16; x <<= 1) mt = fmaxf(mt, __shfl_xor_sync(kFullMask, mt, x));
      const float m_new = fmaxf(m[a], mt);
      const bool live = m_new != -INFINITY;
      const float alpha = live ? exp2f(m[a] - m_new) : 1.f;
      float ls = 0.f;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const float pv = live ? exp2f(s[a][bb] - m_new) : 0.f;
        Ps[(ty + 16 * a) * C::PLD + tx + 16 * bb] = pv;
        ls += pv;
      }
      l_part[a] = l_part[a] * alpha + ls;
      m[a] = m_new;
#pragma unroll
      for (int c = 0; c < C::DC; ++c) {
        o[a][c].x *= alpha;
        o[a][c].y *= alpha;
        o[a][c].z *= alpha;
        o[a][c].w *= alpha;
      }
    }
    __syncthreads();  // P complete

    // O += P.V for rows ty+16a, columns 4*tx + 64c.
    const float* Vt = Vs + st * C::KV_FLOATS;
#pragma unroll 2
    for (int k = 0; k < C::TK; k += 4) {
      float4 pa[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) pa[a] = *reinterpret_cast<const float4*>(Ps + (ty + 16 * a) * C::PLD + k);
#pragma unroll
      for (int c = 0; c < C::DC; ++c) {
        float4 v[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          v[kk] = *reinterpret_cast<const float4*>(Vt + (k + kk) * C::LD + 4 * tx + 64 * c);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float pk[4] = {pa[a].x, pa[a].y, pa[a].z, pa[a].w};
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            o[a][c].x = fmaf(pk[kk], v[kk].x, o[a][c].x);
            o[a][c].y = fmaf(pk[kk], v[kk].y, o[a][c].y);
            o[a][c].z = fmaf(pk[kk], v[kk].z, o[a][c].z);
            o[a][c].w = fmaf(pk[kk], v[kk].w, o[a][c].w);
          }
        }
      }
    }
    __syncthreads();  // stage st and P free for reuse
  }

  // Denominators (sum over the 16 tx threads of a row) and output.
  float* og = static_cast<float*>(p.out);
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    float l = l_part[a];
#pragma unroll
    for (int x = 1; x < 16; x <<= 1) l += __shfl_xor_sync(kFullMask, l, x);
    const int t = t0 + ty + 16 * a;
    if (t < p.T && nsplit > 1) {
      const int64_t slot = (((int64_t)b * p.H + h) * p.T + t) * p.nsplit_max + split;
#pragma unroll
      for (int c = 0; c < C::DC; ++c)
        *reinterpret_cast<float4*>(p.part_o + slot * D + 4 * tx + 64 * c) = o[a][c];
      if (tx == 0) {
        p.part_ml[2 * slot] = m[a];
        p.part_ml[2 * slot + 1] = l;
      }
    } else if (t < p.T) {
      const float inv = 1.f / fmaxf(l, 1e-9f);
      float* orow = og + (int64_t)b * p.so_b + (int64_t)h * p.so_h + (int64_t)t * p.so_t;
#pragma unroll
      for (int c = 0; c < C::DC; ++c) {
        const float4 v = make_float4(o[a][c].x * inv, o[a][c].y * inv, o[a][c].z * inv, o[a][c].w * inv);
        if ((reinterpret_cast<uintptr_t>(orow) & 15) == 0) {
          *reinterpret_cast<float4*>(orow + 4 * tx + 64 * c) = v;
        } else {
          orow[4 * tx + 64 * c] = v.x;
          orow[4 * tx + 64 * c + 1] = v.y;
          orow[4 * tx + 64 * c + 2] = v.z;
          orow[4 * tx + 64 * c + 3] = v.w;
        }
      }
    }
  }
}

// Pools are contiguous and 16-byte aligned (validated at the ABI), so every
// 16-byte chunk of a page row is a valid cp.async source.
template <int D, int BS>
int launch_prefill_f32_tiled(const AttnArgs& a, cudaStream_t stream) {
  using C = PfF32Cfg<D>;
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
  const PrefillPlan plan = make_prefill_plan_f32_tiled(a.B, a.H, a.T, a.D, a.max_pages, BS);
  p.kt_per_split = plan.kt_per_split;
  p.nsplit_max = plan.nsplit_max;
  p.part_o = nullptr;
  p.part_ml = nullptr;
  p.run_if = nullptr;
  p.run_epoch = 0;
  if (plan.bytes > 0) {
    if (!a.workspace || a.workspace_bytes < plan.bytes)
      return set_error(B2PA_ERR_WORKSPACE, "paged_prefill: workspace of %zu bytes, %zu needed", a.workspace_bytes,
                       plan.bytes);
    p.part_ml = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + plan.off_part_ml);
    p.part_o = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + plan.off_part_o);
  }
  const size_t smem = C::BYTES;
  if (smem > (size_t)device_max_smem_optin())
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_prefill: %zu bytes of shared memory exceed the device limit", smem);
  auto kern = paged_prefill_f32_tiled_kernel<D, BS>;
  int rc_attr = set_max_dynamic_smem_cached(reinterpret_cast<const void*>(kern), (int)smem);
  if (rc_attr != B2PA_OK) return rc_attr;
  dim3 grid(((a.T + C::TQ - 1) / C::TQ) * plan.nsplit_max, a.H, a.B);
  kern<<<grid, C::THREADS, smem, stream>>>(p);
  if (plan.nsplit_max > 1) {
    PfTcParams pc = {};
    pc.seq_lens = a.seq_lens;
    pc.cur_lens = a.cur_lens;
    pc.max_pages = a.max_pages;
    pc.out = a.out;
    pc.so_b = a.so[0];
    pc.so_h = a.so[1];
    pc.so_t = a.so[2];
    pc.B = a.B;
    pc.H = a.H;
    pc.T = a.T;
    pc.kt_per_split = plan.kt_per_split;
    pc.nsplit_max = plan.nsplit_max;
    pc.bm = C::TQ;
    pc.part_o = p.part_o;
    pc.part_ml = p.part_ml;
    const int64_t rows = (int64_t)a.B * a.H * a.T;
    prefill_combine_kernel<float, D, BS><<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(pc);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_prefill launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

}  // namespace b2pa
