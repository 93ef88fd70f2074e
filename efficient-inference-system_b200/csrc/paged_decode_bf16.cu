// paged_decode_bf16.cu -- bf16 instantiations of the paged decode kernels.
#include "paged_decode.cuh"

namespace b2pa {
int launch_paged_decode_bf16(const AttnArgs& a, const DecodePlan& plan, cudaStream_t s) {
  return dispatch_decode<__nv_bfloat16>(a, plan, s);
}
}  // namespace b2pa
