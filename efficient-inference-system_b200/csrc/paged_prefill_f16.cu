// paged_prefill_f16.cu -- f16 instantiations of the chunked-prefill kernels.
#include "paged_prefill.cuh"

namespace b2pa {
int launch_paged_prefill_f16(const AttnArgs& a, cudaStream_t s) { return dispatch_prefill<__half>(a, s); }
}  // namespace b2pa
