// paged_prefill_bf16.cu -- bf16 instantiations of the chunked-prefill kernels.
#include "paged_prefill.cuh"

namespace b2pa {
int launch_paged_prefill_bf16(const AttnArgs& a, cudaStream_t s) { return dispatch_prefill<__nv_bfloat16>(a, s); }
}  // namespace b2pa
