// paged_prefill_f32.cu -- f32 instantiations of the chunked-prefill kernels:
// the register-tiled kernel for head_dim 64/128, the general one otherwise.
#include "paged_prefill.cuh"
#include "paged_prefill_f32_tiled.cuh"

namespace b2pa {
int launch_paged_prefill_f32(const AttnArgs& a, cudaStream_t s) {
#define B2PA_PF32_CASE(DD, BB) \
  if (a.D == DD && a.block_size == BB) return launch_prefill_f32_tiled<DD, BB>(a, s);
  B2PA_PF32_CASE(64, 8)
  B2PA_PF32_CASE(64, 16)
  B2PA_PF32_CASE(64, 32)
  B2PA_PF32_CASE(128, 8)
  B2PA_PF32_CASE(128, 16)
  B2PA_PF32_CASE(128, 32)
#undef B2PA_PF32_CASE
  return dispatch_prefill<float>(a, s);
}
}  // namespace b2pa
