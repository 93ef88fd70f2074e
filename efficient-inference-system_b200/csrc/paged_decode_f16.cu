// paged_decode_f16.cu -- f16 instantiations of the paged decode kernels.
#include "paged_decode.cuh"

namespace b2pa {
int launch_paged_decode_f16(const AttnArgs& a, const DecodePlan& plan, cudaStream_t s) {
  return dispatch_decode<__half>(a, plan, s);
}
}  // namespace b2pa
