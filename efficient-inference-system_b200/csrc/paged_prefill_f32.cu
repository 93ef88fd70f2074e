// paged_prefill_f32.cu -- f32 instantiations of the chunked-prefill kernels:
// for head_dim 64 the tensor-core kernel on fp16 hi/lo splits of the
// operands (paged_prefill_tc.cuh) backed by the general CUDA-core kernel for
// inputs out of the split's range, for head_dim 128 (or a problem whose split
// copy would not be addressable) the register-tiled CUDA-core kernel, the
// general one otherwise.  The call number that marks the range flag is
// baked into a captured CUDA graph: once a replay has seen an out-of-range
// input, later replays of that graph keep taking the (correct, slower)
// CUDA-core backup.
#include <atomic>

#include "paged_prefill.cuh"
#include "paged_prefill_f32_tiled.cuh"
#include "paged_prefill_tc.cuh"

namespace b2pa {
int launch_paged_prefill_f32(const AttnArgs& a, cudaStream_t s) {
  const PrefillPlan plan = make_prefill_plan(a.B, a.H, a.T, a.D, a.max_pages, a.block_size, a.dtype);
  if (plan.split_tc) {
    // the tensor-core pass, then the general CUDA-core kernel as a backup
    // that redoes the call only if an input was out of the fp16 split's range
    static std::atomic<uint32_t> calls{0};
    const uint32_t epoch = calls.fetch_add(1, std::memory_order_relaxed) * 2654435761u + 0x9e3779b9u;
    const uint32_t* flag = reinterpret_cast<const uint32_t*>(static_cast<const char*>(a.workspace) + plan.off_flag);
#define B2PA_PF32_TC_CASE(BB)                                                 \
    if (a.D == 64 && a.block_size == BB) {                                    \
      const int rc = launch_prefill_tc<float, 64, BB>(a, s, epoch);           \
      if (rc != B2PA_OK) return rc;                                           \
      return launch_prefill_simt<float, 64, BB>(a, s, flag, epoch);           \
    }
    B2PA_PF32_TC_CASE(8)
    B2PA_PF32_TC_CASE(16)
    B2PA_PF32_TC_CASE(32)
#undef B2PA_PF32_TC_CASE
  }
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
