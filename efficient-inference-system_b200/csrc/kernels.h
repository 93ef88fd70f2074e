// kernels.h -- host-side launcher interface between the C ABI (abi.cu) and
// the kernel translation units.  Arguments are validated by abi.cu before a
// launcher runs; launchers return a b2pa_status and record details through
// set_error().
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "b2pa.h"

namespace b2pa {

// Records a formatted error message for b2pa_last_error_string() and returns
// `code` so callers can `return set_error(code, ...)`.
int set_error(int code, const char* fmt, ...);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per kernel and
// device (the call costs microseconds; launches are hot).
int set_max_dynamic_smem_cached(const void* func, int bytes);

// Multiprocessor count of the current device (cached per device).
int device_sm_count();

// Launches `kern` with programmatic stream serialization: it may begin while
// the previous kernel in `stream` is still running and must call pdl_wait()
// (common.cuh) before reading that kernel's results.  Host-only helper.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Largest dynamic shared memory per block on the current device (opt-in).
int device_max_smem_optin();

struct AppendArgs {
  const void* k_new;
  const void* v_new;
  int64_t sk[4];  // k_new element strides [B,H,T,D]
  int64_t sv[4];  // v_new element strides
  void* k_pool;
  void* v_pool;
  int64_t num_blocks;
  const int32_t* page_table;
  int64_t pt_stride;
  int max_pages;
  const int32_t* start_pos;
  const int32_t* lengths;
  int B, H, T, D, block_size, dtype;
  int32_t* status;
};

struct ZeroArgs {
  void* k_pool;
  void* v_pool;
  int64_t num_blocks;
  const int32_t* block_ids;
  int n_ids;
  int H, D, block_size, dtype;
  int32_t* status;
};

struct AttnArgs {
  const void* q;
  int64_t sq[4];  // q element strides [B,H,T,D]
  const void* k_pool;
  const void* v_pool;
  int64_t num_blocks;
  const int32_t* page_table;
  int64_t pt_stride;
  int max_pages;
  const int32_t* seq_lens;
  const int32_t* cur_lens;
  void* out;
  int64_t so[4];  // out element strides
  int B, H, T, D, block_size, dtype;
  float scale;
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;
  // KV append fused into the attention launch (b2pa_paged_decode_append,
  // b2pa_paged_prefill_append); unused when app_len is null.  For each b,
  // rows t < min(app_len[b], T) of k_new/v_new ([B,H,T,D], element strides
  // skn/svn of B, H and T, unit D stride) are written at positions
  // app_start[b] + t; app_vb is the byte width of the decode's row copy.
  // seq_out (optional) receives seq_lens as int64.
  const void* k_new;
  const void* v_new;
  int64_t skn[3], svn[3];
  const int32_t* app_start;
  const int32_t* app_len;
  int app_vb;
  int64_t* seq_out;
  // The kernel before the attention in the stream is b2pa's append kernel,
  // which waits for its own predecessors before it lets dependents launch:
  // everything but the pool pages it writes is complete when the attention
  // starts, so the attention may set up (and read q and the table) before
  // waiting for it.
  int after_append;
};

int launch_kv_append(const AppendArgs& a, cudaStream_t stream);
int launch_copy_lengths(const int32_t* seq_lens, int64_t* out, int B, cudaStream_t stream);
int launch_zero_blocks(const ZeroArgs& a, cudaStream_t stream);
int launch_patch_table(int32_t* table, int64_t n_cells, const int32_t* pairs, int n_pairs, int32_t* status,
                       cudaStream_t stream);

// Contiguous decode split: a CTA takes at least kDecodeMinUnits pages, and
// the launch is capped at kDecodeMaxCtasPerSm CTAs per SM (two partial slots
// each in the workspace).
// The plan takes it from kDecodeContigStreamsPerSm head-group streams per SM.
constexpr int kDecodeMinUnits = 4;
constexpr int kDecodeMaxCtasPerSm = 8;
constexpr int kDecodeContigStreamsPerSm = 3;

// Decode planning shared by the workspace query and the launcher.
struct DecodePlan {
  int G;                // heads per CTA (consumer warps)
  int HG;               // head groups = H / G
  int pages_per_split;  // P (item split)
  int contig;           // 1: contiguous split (per-CTA ranges of pages)
  int64_t max_items;    // upper bound on work items (contiguous split: partial slots)
  size_t off_item_off, off_part_ml, off_part_acc, bytes;
};
DecodePlan make_decode_plan(int B, int H, int D, int max_pages, int block_size, int dtype);

int launch_paged_decode_f32(const AttnArgs& a, const DecodePlan& plan, cudaStream_t s);
int launch_paged_decode_bf16(const AttnArgs& a, const DecodePlan& plan, cudaStream_t s);
int launch_paged_decode_f16(const AttnArgs& a, const DecodePlan& plan, cudaStream_t s);

// Key-range split of the tensor-core prefill (shared by the workspace query
// and the launcher).  bytes == 0 means no split and no workspace.
struct PrefillPlan {
  int bm;            // query rows per CTA (128: tensor-core kernel, 64: fp32 tiled kernel)
  int kt_per_split;  // 64-key tiles per CTA
  int nsplit_max;
  int split_tc;      // fp32 on the tensor cores: pages split into fp16 hi/lo in the workspace
  // split_tc: split pages, slot table and the out-of-range flag
  size_t off_part_ml, off_part_o, off_split_k, off_split_v, off_slots, off_flag, bytes;
};
PrefillPlan make_prefill_plan(int B, int H, int T, int D, int max_pages, int block_size, int dtype);
// The fp32 register-tiled kernel's plan (its workspace offsets from 0).
PrefillPlan make_prefill_plan_f32_tiled(int B, int H, int T, int D, int max_pages, int block_size);
bool prefill_uses_tensor_cores(int D, int block_size, int dtype, int64_t pool_rows);

int launch_paged_prefill_f32(const AttnArgs& a, cudaStream_t s);
int launch_paged_prefill_bf16(const AttnArgs& a, cudaStream_t s);
int launch_paged_prefill_f16(const AttnArgs& a, cudaStream_t s);

inline int dtype_size(int dtype) {
  return dtype == B2PA_DTYPE_F32 ? 4 : (dtype == B2PA_DTYPE_BF16 || dtype == B2PA_DTYPE_F16) ? 2 : 0;
}

inline bool head_dim_supported(int D) { return D == 16 || D == 32 || D == 64 || D == 128 || D == 256; }
inline bool block_size_supported(int bs) { return bs == 8 || bs == 16 || bs == 32; }

}  // namespace b2pa
