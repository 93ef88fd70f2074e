// selftest.cu -- exercises the kernels' bounded-wait failure path on a GPU
// without faulting it.
//
// Every spin-wait in the b2pa kernels (mbarrier waits of the decode ring and
// of the tcgen05 prefill pipeline) gives up after kWaitLimitNs of
// %globaltimer, records B2PA_ERR_DEVICE_TIMEOUT in the status word and lets
// the kernel return.  With valid inputs those waits always complete, so the
// give-up path cannot be reached through the attention entry points.  This
// kernel reaches it on purpose: one warp waits, through the same
// mbar_wait_bounded, on an mbarrier that nothing ever arrives at.  The wait
// ends after the limit, the status word says so and the CUDA context stays
// usable -- what a test of the timeout path needs.  No reference counterpart.
#include "b2pa.h"
#include "common.cuh"
#include "kernels.h"

namespace b2pa {

__global__ void __launch_bounds__(32) selftest_wait_timeout_kernel(int32_t* status, int32_t* done) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none ever comes
    fence_mbar_init();
  }
  __syncwarp();
  const bool ok = __all_sync(kFullMask, mbar_wait_bounded(&bar, 0, status));
  if (threadIdx.x == 0) *done = ok ? 1 : 2;  // 2: the wait gave up and the kernel went on
}

int launch_selftest_wait_timeout(int32_t* status, int32_t* done, cudaStream_t stream) {
  selftest_wait_timeout_kernel<<<1, 32, 0, stream>>>(status, done);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "selftest_wait_timeout launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

}  // namespace b2pa

extern "C" int b2pa_selftest_wait_timeout(int32_t* status, int32_t* done, void* stream) {
  if (!status || !done) return b2pa::set_error(B2PA_ERR_INVALID_ARGUMENT, "selftest_wait_timeout: null pointer");
  return b2pa::launch_selftest_wait_timeout(status, done, static_cast<cudaStream_t>(stream));
}
