// paged_decode_noalloc.cu -- b2pa_paged_decode for callers that cannot
// allocate device memory.
//
// b2pa_paged_decode needs scratch space (the split plan and the split-K
// partials) and asks the caller to pass it in.  Some callers have no way to
// provide it: code that runs where cudaMalloc is off limits (a host callback
// or a real-time thread that must not block on the allocator, a plugin whose
// host framework owns all device memory and hands out only the tensors of
// the call, or a process that must not grow its footprint after start-up).
// For them this file keeps the scratch in a fixed array that lives in the
// library itself: b2pa_paged_decode_noalloc takes the same inputs and output
// as b2pa_paged_decode, minus the workspace, and allocates nothing.
//
// Limits and sharing rules (also stated in b2pa.h):
//   * the array holds B2PA_NOALLOC_SCRATCH_BYTES (32 MiB).  Every GPU that
//     loads libb2pa.so holds that much device memory until the process exits.
//     A problem whose plan needs more is rejected with B2PA_ERR_WORKSPACE
//     before anything is launched; use b2pa_paged_decode for those.
//   * all calls on a device share the one array, and it keeps whatever the
//     last call left in it.  Nothing in it has to start at zero: every call
//     writes the plan and every partial before reading them.  Two calls whose
//     kernels overlap on the GPU (different streams, no ordering between
//     them) race on the array and produce garbage; order such calls on one
//     stream or with events.
//   * the first call in each CUDA context looks up the array's device address
//     with cudaGetSymbolAddress, which makes the CUDA runtime load this module
//     on that device.  Make that first call outside any stream capture (a
//     warm-up call at start-up is enough); a first call on a capturing stream
//     returns B2PA_ERR_UNSUPPORTED.  Later calls in the same context read the
//     cached address; a new context on the device (cudaDeviceReset, or the
//     primary context released and created again) counts as a first call.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "b2pa.h"
#include "kernels.h"

namespace b2pa {
namespace {

constexpr size_t kScratchBytes = (size_t)B2PA_NOALLOC_SCRATCH_BYTES;

// The scratch array.  Host code must not use &g_noalloc_scratch as a device
// address (on the host it names a shadow variable); it goes through
// scratch_address() below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
// Per device: the array's address and the id of the context it was looked up
// in.  A context created anew on that device (after cudaDeviceReset, or after
// the primary context was released and retained again) has another id, so the
// address is looked up again instead of reusing one that no longer exists.
struct CachedAddress {
  unsigned long long ctx_id;
  void* addr;
};
CachedAddress g_addr[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <typename Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
    return reinterpret_cast<Fn>(p);
  return nullptr;
}

// Identifies the current context: its process-unique id (cuCtxGetId), or its
// handle where the driver lacks that call.
int current_context_id(unsigned long long* id) {
  static std::once_flag once;
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  std::call_once(once, [] {
    get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
    get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  });
  if (get_current == nullptr)
    return set_error(B2PA_ERR_CUDA, "paged_decode_noalloc: the driver has no cuCtxGetCurrent");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    return set_error(B2PA_ERR_CUDA, "paged_decode_noalloc: no current CUDA context");
  unsigned long long v = 0;
  if (get_id == nullptr || get_id(ctx, &v) != CUDA_SUCCESS) v = (unsigned long long)(uintptr_t)ctx;
  *id = v;
  return B2PA_OK;
}

// Device address of g_noalloc_scratch in the current context; looked up once
// per context with its device current.  The look-up may load this module on
// the device, which must not happen inside a stream capture: a first call
// that finds `stream` capturing is refused.
int scratch_address(cudaStream_t stream, void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode_noalloc: device %d out of range", dev);
  unsigned long long ctx_id = 0;
  const int rc = current_context_id(&ctx_id);
  if (rc != B2PA_OK) return rc;
  std::lock_guard<std::mutex> g(g_mu);
  if (g_addr[dev].addr == nullptr || g_addr[dev].ctx_id != ctx_id) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess || cap != cudaStreamCaptureStatusNone)
      return set_error(B2PA_ERR_UNSUPPORTED,
                       "paged_decode_noalloc: the first call in a CUDA context looks up the scratch array and "
                       "cannot run inside a stream capture; make one call before capturing");
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(B2PA_ERR_CUDA, "paged_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_addr[dev].addr = p;
    g_addr[dev].ctx_id = ctx_id;
  }
  *out = g_addr[dev].addr;
  return B2PA_OK;
}

}  // namespace
}  // namespace b2pa

extern "C" int b2pa_paged_decode_noalloc(const void* q, const int64_t q_strides[4], const void* k_pool,
                                         const void* v_pool, const int64_t pool_strides[4], int64_t num_blocks,
                                         const int32_t* page_table, int64_t pt_stride, int max_pages,
                                         const int32_t* seq_lens, const int32_t* cur_lens, void* out,
                                         const int64_t out_strides[4], int B, int H, int D, int block_size,
                                         float scale, int dtype, int32_t* status, void* stream) {
  using namespace b2pa;
  // Same size check the workspace query uses; reject before touching the GPU.
  if (B > 0 && H > 0 && D > 0 && max_pages >= 0 && block_size > 0 && dtype_size(dtype) != 0) {
    const size_t need = b2pa_paged_decode_workspace_size(B, H, D, max_pages, block_size, dtype);
    if (need > kScratchBytes)
      return set_error(B2PA_ERR_WORKSPACE,
                       "paged_decode_noalloc: this problem needs %zu bytes of scratch but the built-in array holds "
                       "%zu; call b2pa_paged_decode with a workspace instead",
                       need, kScratchBytes);
  }
  void* scratch = nullptr;
  if (B > 0) {
    const int rc = scratch_address(static_cast<cudaStream_t>(stream), &scratch);
    if (rc != B2PA_OK) return rc;
  }
  return b2pa_paged_decode(q, q_strides, k_pool, v_pool, pool_strides, num_blocks, page_table, pt_stride, max_pages,
                           seq_lens, cur_lens, out, out_strides, B, H, D, block_size, scale, dtype, scratch,
                           kScratchBytes, status, stream);
}
