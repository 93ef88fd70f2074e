// common.cuh -- shared device helpers for the b2pa kernels (sm_100a only).
//
// Contents: element-type traits and 4/8/16-byte vector conversions, the
// device status word, and thin inline-PTX wrappers for mbarriers and the
// (non-multicast) bulk copy global -> shared.  Every wait in these kernels is
// bounded by a wall-clock limit read from %globaltimer; a wait that gives up
// records B2PA_ERR_DEVICE_TIMEOUT in the status word and returns false.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "b2pa.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "b2pa kernels target sm_100a (B200) only"
#endif

namespace b2pa {

constexpr unsigned kFullMask = 0xffffffffu;
// Bounded waits give up after this many nanoseconds (one second).
constexpr uint64_t kWaitLimitNs = 1000000000ull;
constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------- status ---
__device__ __forceinline__ void set_status(int32_t* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------ type traits ---
template <typename T> struct ElemTraits;
template <> struct ElemTraits<float> { static constexpr int kDtype = B2PA_DTYPE_F32; };
template <> struct ElemTraits<__nv_bfloat16> { static constexpr int kDtype = B2PA_DTYPE_BF16; };
template <> struct ElemTraits<__half> { static constexpr int kDtype = B2PA_DTYPE_F16; };

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Unpack one 32-bit word holding two 16-bit elements into floats.
__device__ __forceinline__ float2 unpack2(uint32_t w, __nv_bfloat16*) {
  // bf16 -> f32 is exact: the bf16 bits are the top half of the f32 bits.
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ float2 unpack2(uint32_t w, __half*) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}

// Vector of N elements of T moved as one aligned access of N*sizeof(T) bytes
// (4, 8 or 16 bytes).
template <int BYTES> struct VecWord;
template <> struct VecWord<4> { using type = uint32_t; };
template <> struct VecWord<8> { using type = uint2; };
template <> struct VecWord<16> { using type = uint4; };

template <typename T, int N>
struct Vec {
  static constexpr int kBytes = N * (int)sizeof(T);
  using Word = typename VecWord<kBytes>::type;
  Word w;

  __device__ __forceinline__ void to_float(float* f) const {
    if constexpr (sizeof(T) == 4) {
      const float* p = reinterpret_cast<const float*>(&w);
#pragma unroll
      for (int i = 0; i < N; ++i) f[i] = p[i];
    } else {
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&w);
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        float2 v = unpack2(p[i], static_cast<T*>(nullptr));
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
      }
    }
  }

  // 16-bit types convert two values per instruction (round to nearest,
  // the same bits as two single conversions).
  __device__ __forceinline__ void from_float(const float* f) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
      for (int i = 0; i < N / 2; ++i) p[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    } else if constexpr (std::is_same<T, __half>::value) {
      __half2* p = reinterpret_cast<__half2*>(&w);
#pragma unroll
      for (int i = 0; i < N / 2; ++i) p[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    } else {
      T* p = reinterpret_cast<T*>(&w);
#pragma unroll
      for (int i = 0; i < N; ++i) p[i] = from_f32<T>(f[i]);
    }
  }
};

template <typename W>
__device__ __forceinline__ W ld_shared(const void* p) {
  return *reinterpret_cast<const W*>(p);
}

// Streaming global load (read once, do not keep in L1).
template <typename W>
__device__ __forceinline__ W ld_global_nc(const void* p) {
  return __ldg(reinterpret_cast<const W*>(p));
}

// ------------------------------------------------------------- mbarriers ---
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Orders this thread's earlier generic-proxy global stores before its later
// async-proxy accesses (bulk copies) of the same global memory.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Makes mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

// Raises the barrier's expected transaction bytes without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits until the phase with the given parity has completed.  Gives up after
// kWaitLimitNs, records B2PA_ERR_DEVICE_TIMEOUT and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) {
      set_status(status, B2PA_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
}

// One-dimensional bulk copy global -> this CTA's shared memory, completing
// `bytes` transactions on `bar`.  No multicast.  dst, src 16-byte aligned and
// bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2^x with the hardware approximation (PTX ex2.approx.ftz.f32: relative
// error about 2^-22, subnormal results flushed to zero), for softmax weights.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Maximum of three fp32 values in one instruction (sm_100 `max.f32` with
// three sources); exact, like two fmaxf.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Packed two-lane fp32 arithmetic of sm_100 (one instruction for two
// values): d = a * b + c and d = a + b, each lane rounded to nearest.
__device__ __forceinline__ uint64_t f2_bits(float2 v) {
  return (uint64_t)__float_as_uint(v.x) | ((uint64_t)__float_as_uint(v.y) << 32);
}
__device__ __forceinline__ float2 f2_from_bits(uint64_t b) {
  return make_float2(__uint_as_float((uint32_t)b), __uint_as_float((uint32_t)(b >> 32)));
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return f2_from_bits(d);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from_bits(d);
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while its predecessor in the stream is still
// running.  pdl_wait() returns once the predecessor grid has completed and
// its memory is visible (a no-op for a normal launch); every kernel below
// calls it before touching memory an earlier kernel may write.
// pdl_launch_dependents() lets the successor start launching early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------ warp utils ---
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(kFullMask, v, m));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(kFullMask, v, m);
  return v;
}

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x / 2); }

}  // namespace b2pa
