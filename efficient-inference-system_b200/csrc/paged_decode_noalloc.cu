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
//   * the first call on each device looks up the array's device address with
//     cudaGetSymbolAddress, which makes the CUDA runtime load this module on
//     that device.  Make that first call outside any stream capture (a warm-up
//     call at start-up is enough); later calls only read the cached address.
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
void* g_addr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device; looked up once
// per device with that device current.
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> g(g_mu);
  if (g_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(B2PA_ERR_CUDA, "paged_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
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
    const int rc = scratch_address(&scratch);
    if (rc != B2PA_OK) return rc;
  }
  return b2pa_paged_decode(q, q_strides, k_pool, v_pool, pool_strides, num_blocks, page_table, pt_stride, max_pages,
                           seq_lens, cur_lens, out, out_strides, B, H, D, block_size, scale, dtype, scratch,
                           kScratchBytes, status, stream);
}
