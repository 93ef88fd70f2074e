// paged_prefill_f32.cu -- f32 instantiations of the chunked-prefill kernels.
#include "paged_prefill.cuh"

namespace b2pa {
int launch_paged_prefill_f32(const AttnArgs& a, cudaStream_t s) { return dispatch_prefill<float>(a, s); }
}  // namespace b2pa
