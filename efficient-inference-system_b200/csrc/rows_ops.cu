// rows_ops.cu -- the non-attention operations of a decode step, fp32, for a
// few rows (the batch's new tokens: M <= 16).
//
// In a decode step of the reference's model (src/model/transformer.py:7-35,
// 133-181; src/model/attention.py:46-48,63-64) every matrix product has only
// M = batch rows, so each is a matrix-vector product bound by reading the
// weights once from HBM, and each LayerNorm, bias, GELU and residual add is
// its own small launch in torch.  Here one kernel does
//   y = act(LN(x) . W^T + bias)   or   y += LN(x) . W^T + bias
// for all M rows: the (normalised) rows sit in shared memory, and each warp
// streams whole weight rows (coalesced 16-byte loads, no L1 allocation) and
// dots them against every staged row, so the weights are read exactly once.
// Two more kernels gather the token + position embeddings and take the
// argmax over the vocabulary.  All are launched as programmatic dependents:
// they wait for the kernel before them before reading its results (the
// linear kernel requests the first pieces of its weight rows before waiting,
// since the weights never depend on that kernel).
//
// Numerics: fp32 throughout, FMA accumulation; LayerNorm as torch computes it
// (biased variance, rsqrt(var + eps)); GELU exact, 0.5 x (1 + erf(x / sqrt 2)),
// as nn.GELU(); argmax returns the first index of the maximum, as
// torch.argmax.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace b2pa {
namespace {

constexpr int kRowsWarps = 4;     // warps per CTA; one output column (weight row) per warp
constexpr int kRowsMaxM = 16;     // rows per call
constexpr int kRowsMaxElems = 32768;  // M * K staged in shared memory (128 KB)

struct RowsLinearArgs {
  const float* x;
  int64_t xs;
  int M, K, N;
  const float* ln_w;
  const float* ln_b;
  float eps;
  const float* w;
  const float* bias;
  int act;         // 0: none, 1: GELU (erf)
  float* y;
  int64_t ys;
  int accumulate;  // y += result
};

__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

template <int MAXM>
__global__ void __launch_bounds__(kRowsWarps * 32) rows_linear_kernel(RowsLinearArgs a) {
  extern __shared__ float4 xs4[];  // [M][K/4]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K4 = a.K >> 2;
  const int M = a.M;
  const int n = blockIdx.x * kRowsWarps + warp;
  const bool active = n < a.N;
  const float4* wrow = reinterpret_cast<const float4*>(a.w + (int64_t)(active ? n : 0) * a.K);
  // The weights do not depend on the kernel before this one: the first 128
  // 16-byte pieces of this warp's weight row are requested before waiting
  // for it, so their latency overlaps its tail.
  float4 w0[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int k = lane + 32 * u;
    w0[u] = (active && k < K4) ? ld_stream(wrow + k) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  pdl_wait();
  pdl_launch_dependents();
  for (int i = tid; i < M * K4; i += blockDim.x) {
    const int m = i / K4, k4 = i - m * K4;
    xs4[i] = *reinterpret_cast<const float4*>(a.x + (int64_t)m * a.xs + 4 * k4);
  }
  __syncthreads();
  if (a.ln_w != nullptr) {
    // LayerNorm of each row in place: a warp per row, two passes (mean, then
    // the biased variance of the centred values)
    for (int m = warp; m < M; m += kRowsWarps) {
      float4* row = xs4 + (int64_t)m * K4;
      float s = 0.f;
      for (int k4 = lane; k4 < K4; k4 += 32) {
        const float4 v = row[k4];
        s += (v.x + v.y) + (v.z + v.w);
      }
      const float mean = warp_sum(s) / (float)a.K;
      float q = 0.f;
      for (int k4 = lane; k4 < K4; k4 += 32) {
        const float4 v = row[k4];
        const float dx = v.x - mean, dy = v.y - mean, dz = v.z - mean, dw = v.w - mean;
        q += (dx * dx + dy * dy) + (dz * dz + dw * dw);
      }
      const float rstd = rsqrtf(warp_sum(q) / (float)a.K + a.eps);
      for (int k4 = lane; k4 < K4; k4 += 32) {
        const float4 v = row[k4];
        const float4 g = reinterpret_cast<const float4*>(a.ln_w)[k4];
        const float4 b = a.ln_b != nullptr ? reinterpret_cast<const float4*>(a.ln_b)[k4] : make_float4(0, 0, 0, 0);
        row[k4] = make_float4((v.x - mean) * rstd * g.x + b.x, (v.y - mean) * rstd * g.y + b.y,
                              (v.z - mean) * rstd * g.z + b.z, (v.w - mean) * rstd * g.w + b.w);
      }
    }
    __syncthreads();
  }
  if (!active) return;
  float acc[MAXM];
#pragma unroll
  for (int m = 0; m < MAXM; ++m) acc[m] = 0.f;
  // the prefetched pieces, then four loads in flight per lane at a time
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int k = lane + 32 * u;
    if (k < K4) {
#pragma unroll
      for (int m = 0; m < MAXM; ++m) {
        if (m < M) {
          const float4 xv = xs4[(int64_t)m * K4 + k];
          acc[m] = fmaf(w0[u].x, xv.x, fmaf(w0[u].y, xv.y, fmaf(w0[u].z, xv.z, fmaf(w0[u].w, xv.w, acc[m]))));
        }
      }
    }
  }
  int k4 = lane + 128;
  for (; k4 + 96 < K4; k4 += 128) {
    float4 w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w[u] = ld_stream(wrow + k4 + 32 * u);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
      for (int m = 0; m < MAXM; ++m) {
        if (m < M) {
          const float4 xv = xs4[(int64_t)m * K4 + k4 + 32 * u];
          acc[m] = fmaf(w[u].x, xv.x, fmaf(w[u].y, xv.y, fmaf(w[u].z, xv.z, fmaf(w[u].w, xv.w, acc[m]))));
        }
      }
    }
  }
  for (; k4 < K4; k4 += 32) {
    const float4 w = ld_stream(wrow + k4);
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
      if (m < M) {
        const float4 xv = xs4[(int64_t)m * K4 + k4];
        acc[m] = fmaf(w.x, xv.x, fmaf(w.y, xv.y, fmaf(w.z, xv.z, fmaf(w.w, xv.w, acc[m]))));
      }
    }
  }
  const float bn = a.bias != nullptr ? a.bias[n] : 0.f;
#pragma unroll
  for (int m = 0; m < MAXM; ++m) {
    if (m < M) {
      float v = warp_sum(acc[m]) + bn;
      if (a.act == 1) v = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
      if (lane == m % 32) {
        float* dst = a.y + (int64_t)m * a.ys + n;
        *dst = a.accumulate ? *dst + v : v;
      }
    }
  }
}

// x[m, :] = token_table[ids[m], :] + position_table[pos[m], :]
__global__ void __launch_bounds__(128) rows_embed_kernel(const int64_t* ids, const int64_t* pos, int M,
                                                         const float* tok, int64_t vocab, const float* pe,
                                                         int64_t max_pos, int K, float* x, int64_t xs,
                                                         int32_t* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int m = blockIdx.x;
  if (m >= M) return;
  const int64_t t = ids[m], p = pos[m];
  const bool ok = t >= 0 && t < vocab && p >= 0 && p < max_pos;
  if (!ok && threadIdx.x == 0) set_status(status, B2PA_ERR_INVALID_ARGUMENT);
  const float4* a4 = reinterpret_cast<const float4*>(tok + (ok ? t : 0) * K);
  const float4* b4 = reinterpret_cast<const float4*>(pe + (ok ? p : 0) * K);
  float4* o4 = reinterpret_cast<float4*>(x + (int64_t)m * xs);
  for (int k4 = threadIdx.x; k4 < K / 4; k4 += blockDim.x) {
    const float4 u = a4[k4], v = b4[k4];
    o4[k4] = ok ? make_float4(u.x + v.x, u.y + v.y, u.z + v.z, u.w + v.w) : make_float4(0, 0, 0, 0);
  }
}

// out[m] = the first index of the largest x[m, :]
__global__ void __launch_bounds__(256) rows_argmax_kernel(const float* x, int64_t xs, int M, int N, int64_t* out) {
  pdl_wait();
  pdl_launch_dependents();
  const int m = blockIdx.x;
  if (m >= M) return;
  const float* row = x + (int64_t)m * xs;
  float best = -INFINITY;
  int idx = N;  // no element seen yet
  for (int n = threadIdx.x; n < N; n += blockDim.x) {
    const float v = row[n];
    if (v > best || (idx == N && !(v < best))) {  // first strict maximum of this thread's columns
      best = v;
      idx = n;
    }
  }
  // reduce (value, index): larger value wins, equal values keep the smaller index
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float bv = __shfl_xor_sync(kFullMask, best, o);
    const int bi = __shfl_xor_sync(kFullMask, idx, o);
    if (bv > best || (bv == best && bi < idx)) {
      best = bv;
      idx = bi;
    }
  }
  __shared__ float sv[8];
  __shared__ int si[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < idx)) {
        best = sv[w];
        idx = si[w];
      }
    out[m] = idx < N ? idx : 0;
  }
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace
}  // namespace b2pa

using namespace b2pa;

extern "C" int b2pa_rows_linear(const float* x, int64_t x_row_stride, int M, int K, const float* ln_weight,
                                const float* ln_bias, float ln_eps, const float* weight, const float* bias, int N,
                                int activation, float* y, int64_t y_row_stride, int accumulate, int32_t* status,
                                void* stream) {
  (void)status;
  if (M < 0 || K <= 0 || N <= 0 || M > kRowsMaxM)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "rows_linear: bad sizes M=%d K=%d N=%d (M <= %d)", M, K, N,
                     kRowsMaxM);
  if (M == 0) return B2PA_OK;
  if (!x || !weight || !y) return set_error(B2PA_ERR_INVALID_ARGUMENT, "rows_linear: null pointer argument");
  if (K % 4 || (int64_t)M * K > kRowsMaxElems)
    return set_error(B2PA_ERR_UNSUPPORTED, "rows_linear: K must be a multiple of 4 and M*K <= %d", kRowsMaxElems);
  if (activation != 0 && activation != 1)
    return set_error(B2PA_ERR_UNSUPPORTED, "rows_linear: unknown activation %d", activation);
  if (!aligned16(x) || !aligned16(weight) || x_row_stride % 4 || x_row_stride < K || y_row_stride < N ||
      (ln_weight && !aligned16(ln_weight)) || (ln_bias && !aligned16(ln_bias)))
    return set_error(B2PA_ERR_UNSUPPORTED, "rows_linear: x, weight and LayerNorm vectors need 16-byte rows");
  {
    // every CTA reads all of x while others already write y: they must not overlap
    const uintptr_t x0 = reinterpret_cast<uintptr_t>(x), y0 = reinterpret_cast<uintptr_t>(y);
    const uintptr_t x1 = x0 + 4 * (uintptr_t)((int64_t)(M - 1) * x_row_stride + K);
    const uintptr_t y1 = y0 + 4 * (uintptr_t)((int64_t)(M - 1) * y_row_stride + N);
    if (x0 < y1 && y0 < x1) return set_error(B2PA_ERR_INVALID_ARGUMENT, "rows_linear: y overlaps x");
  }
  RowsLinearArgs a;
  a.x = x;
  a.xs = x_row_stride;
  a.M = M;
  a.K = K;
  a.N = N;
  a.ln_w = ln_weight;
  a.ln_b = ln_bias;
  a.eps = ln_eps;
  a.w = weight;
  a.bias = bias;
  a.act = activation;
  a.y = y;
  a.ys = y_row_stride;
  a.accumulate = accumulate ? 1 : 0;
  const size_t smem = (size_t)M * K * 4;
  const dim3 grid((unsigned)((N + kRowsWarps - 1) / kRowsWarps));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (M == 1) {
    int rc = set_max_dynamic_smem_cached(reinterpret_cast<const void*>(rows_linear_kernel<1>), (int)smem);
    if (rc != B2PA_OK) return rc;
    e = launch_pdl(rows_linear_kernel<1>, grid, dim3(kRowsWarps * 32), smem, s, a);
  } else if (M <= 4) {
    int rc = set_max_dynamic_smem_cached(reinterpret_cast<const void*>(rows_linear_kernel<4>), (int)smem);
    if (rc != B2PA_OK) return rc;
    e = launch_pdl(rows_linear_kernel<4>, grid, dim3(kRowsWarps * 32), smem, s, a);
  } else {
    int rc = set_max_dynamic_smem_cached(reinterpret_cast<const void*>(rows_linear_kernel<kRowsMaxM>), (int)smem);
    if (rc != B2PA_OK) return rc;
    e = launch_pdl(rows_linear_kernel<kRowsMaxM>, grid, dim3(kRowsWarps * 32), smem, s, a);
  }
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "rows_linear launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

extern "C" int b2pa_rows_embed(const int64_t* token_ids, const int64_t* positions, int M, const float* token_table,
                               int64_t vocab, const float* position_table, int64_t max_positions, int K, float* x,
                               int64_t x_row_stride, int32_t* status, void* stream) {
  if (M < 0 || K <= 0 || vocab <= 0 || max_positions <= 0)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "rows_embed: bad sizes");
  if (M == 0) return B2PA_OK;
  if (!token_ids || !positions || !token_table || !position_table || !x)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "rows_embed: null pointer argument");
  if (K % 4 || x_row_stride % 4 || x_row_stride < K || !aligned16(token_table) || !aligned16(position_table) ||
      !aligned16(x))
    return set_error(B2PA_ERR_UNSUPPORTED, "rows_embed: tables and x need 16-byte rows");
  cudaError_t e = launch_pdl(rows_embed_kernel, dim3((unsigned)M), dim3(128), 0, static_cast<cudaStream_t>(stream),
                             token_ids, positions, M, token_table, vocab, position_table, max_positions, K, x,
                             x_row_stride, status);
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "rows_embed launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

extern "C" int b2pa_rows_argmax(const float* x, int64_t x_row_stride, int M, int N, int64_t* out, int32_t* status,
                                void* stream) {
  (void)status;
  if (M < 0 || N <= 0 || x_row_stride < N) return set_error(B2PA_ERR_INVALID_ARGUMENT, "rows_argmax: bad sizes");
  if (M == 0) return B2PA_OK;
  if (!x || !out) return set_error(B2PA_ERR_INVALID_ARGUMENT, "rows_argmax: null pointer argument");
  cudaError_t e = launch_pdl(rows_argmax_kernel, dim3((unsigned)M), dim3(256), 0, static_cast<cudaStream_t>(stream),
                             x, x_row_stride, M, N, out);
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "rows_argmax launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}
