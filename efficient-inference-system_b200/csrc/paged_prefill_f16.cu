// paged_prefill_f16.cu -- f16 instantiations of the chunked-prefill kernels:
// tcgen05/TMEM tiles for head_dim 64 and 128, fp32 CUDA-core tiles otherwise.
#include "paged_prefill.cuh"
#include "paged_prefill_tc.cuh"

namespace b2pa {
int launch_paged_prefill_f16(const AttnArgs& a, cudaStream_t s) {
  if (prefill_uses_tensor_cores(a.D, a.block_size, a.dtype, a.num_blocks * a.H * a.block_size)) {
#define B2PA_TC_CASE(DD, BB) \
    if (a.D == DD && a.block_size == BB) return launch_prefill_tc<__half, DD, BB>(a, s);
    B2PA_TC_CASE(64, 8) B2PA_TC_CASE(64, 16) B2PA_TC_CASE(64, 32)
    B2PA_TC_CASE(128, 8) B2PA_TC_CASE(128, 16) B2PA_TC_CASE(128, 32)
#undef B2PA_TC_CASE
  }
  return dispatch_prefill<__half>(a, s);
}
}  // namespace b2pa
