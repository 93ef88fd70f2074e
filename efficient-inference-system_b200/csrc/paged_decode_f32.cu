// paged_decode_f32.cu -- f32 instantiations of the paged decode kernels.
#include "paged_decode.cuh"

namespace b2pa {
int launch_paged_decode_f32(const AttnArgs& a, const DecodePlan& plan, cudaStream_t s) {
  return dispatch_decode<float>(a, plan, s);
}
}  // namespace b2pa
