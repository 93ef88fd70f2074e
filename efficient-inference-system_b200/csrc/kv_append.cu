// kv_append.cu -- fused KV scatter into the paged pools, and batched block
// zeroing.
//
// Reference behaviour (jacobzhang22/efficient-inference-system):
//   PagedKVCacheState.append, src/cache/paged_kv.py:109-120, copies token
//   `offset .. offset+take` of k_new[0] into k_blocks[block_id, :,
//   block_offset:block_offset+take, :] one block at a time, for each request
//   in turn (BatchedPagedKVCache.append_batch, paged_kv.py:165-171).  Block
//   allocation stays on the host; this kernel does every copy of one
//   append_batch call in a single launch: one CTA per (token, sequence), each
//   moving the H x D row of K and of V with 16-byte accesses where the
//   strides allow.  The copy is a raw byte move, so pools are bit-identical
//   to the reference's slice assignment.
//   LayerBlockPool.release_block, paged_kv.py:80-85, zeroes one block of K
//   and V per call; zero_blocks_kernel zeroes a whole list in one launch.
#include "common.cuh"
#include "kernels.h"

namespace b2pa {

template <int VB>
__global__ void __launch_bounds__(128) kv_append_kernel(AppendArgs a, int es) {
  using W = typename VecWord<VB>::type;
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x;
  const int b = blockIdx.y;
  int len = a.lengths[b];
  len = len < a.T ? len : a.T;
  if (t >= len) return;
  const int64_t pos = (int64_t)a.start_pos[b] + t;
  const int64_t page = pos / a.block_size;
  if (pos < 0 || page >= a.max_pages) {
    if (threadIdx.x == 0) set_status(a.status, B2PA_ERR_BAD_BLOCK_ID);
    return;
  }
  const int32_t blk = a.page_table[(int64_t)b * a.pt_stride + page];
  if (blk < 0 || blk >= a.num_blocks) {
    if (threadIdx.x == 0) set_status(a.status, B2PA_ERR_BAD_BLOCK_ID);
    return;
  }
  const int off = (int)(pos - page * a.block_size);
  const int row_bytes = a.D * es;
  const int cph = row_bytes / VB;  // vector words per head row
  const int total = a.H * cph;
  const char* ks = static_cast<const char*>(a.k_new);
  const char* vs = static_cast<const char*>(a.v_new);
  char* kp = static_cast<char*>(a.k_pool);
  char* vp = static_cast<char*>(a.v_pool);
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int h = i / cph;
    const int c = i - h * cph;
    const int64_t src_k = ((int64_t)b * a.sk[0] + (int64_t)h * a.sk[1] + (int64_t)t * a.sk[2]) * es + (int64_t)c * VB;
    const int64_t src_v = ((int64_t)b * a.sv[0] + (int64_t)h * a.sv[1] + (int64_t)t * a.sv[2]) * es + (int64_t)c * VB;
    const int64_t dst = ((((int64_t)blk * a.H + h) * a.block_size + off) * a.D) * es + (int64_t)c * VB;
    const W kw = *reinterpret_cast<const W*>(ks + src_k);
    const W vw = *reinterpret_cast<const W*>(vs + src_v);
    *reinterpret_cast<W*>(kp + dst) = kw;
    *reinterpret_cast<W*>(vp + dst) = vw;
  }
}

// Element-sized copy for 2-byte types whose strides rule out wider words.
__global__ void __launch_bounds__(128) kv_append_kernel_u16(AppendArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x;
  const int b = blockIdx.y;
  int len = a.lengths[b];
  len = len < a.T ? len : a.T;
  if (t >= len) return;
  const int64_t pos = (int64_t)a.start_pos[b] + t;
  const int64_t page = pos / a.block_size;
  if (pos < 0 || page >= a.max_pages) {
    if (threadIdx.x == 0) set_status(a.status, B2PA_ERR_BAD_BLOCK_ID);
    return;
  }
  const int32_t blk = a.page_table[(int64_t)b * a.pt_stride + page];
  if (blk < 0 || blk >= a.num_blocks) {
    if (threadIdx.x == 0) set_status(a.status, B2PA_ERR_BAD_BLOCK_ID);
    return;
  }
  const int off = (int)(pos - page * a.block_size);
  const uint16_t* ks = static_cast<const uint16_t*>(a.k_new);
  const uint16_t* vs = static_cast<const uint16_t*>(a.v_new);
  uint16_t* kp = static_cast<uint16_t*>(a.k_pool);
  uint16_t* vp = static_cast<uint16_t*>(a.v_pool);
  const int total = a.H * a.D;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int h = i / a.D;
    const int d = i - h * a.D;
    const int64_t dst = (((int64_t)blk * a.H + h) * a.block_size + off) * a.D + d;
    kp[dst] = ks[(int64_t)b * a.sk[0] + (int64_t)h * a.sk[1] + (int64_t)t * a.sk[2] + (int64_t)d * a.sk[3]];
    vp[dst] = vs[(int64_t)b * a.sv[0] + (int64_t)h * a.sv[1] + (int64_t)t * a.sv[2] + (int64_t)d * a.sv[3]];
  }
}

template <int VB>
__global__ void __launch_bounds__(256) zero_blocks_kernel(ZeroArgs a, int64_t block_bytes) {
  using W = typename VecWord<VB>::type;
  const int i = blockIdx.x;
  const int32_t blk = a.block_ids[i];
  if (blk < 0 || blk >= a.num_blocks) {
    if (threadIdx.x == 0) set_status(a.status, B2PA_ERR_BAD_BLOCK_ID);
    return;
  }
  char* kp = static_cast<char*>(a.k_pool) + (int64_t)blk * block_bytes;
  char* vp = static_cast<char*>(a.v_pool) + (int64_t)blk * block_bytes;
  W z;
  memset(&z, 0, sizeof(W));
  for (int64_t o = (int64_t)threadIdx.x * VB; o < block_bytes; o += (int64_t)blockDim.x * VB) {
    *reinterpret_cast<W*>(kp + o) = z;
    *reinterpret_cast<W*>(vp + o) = z;
  }
}

// seq_lens as int64 (the lengths append_batch returns), for the fused
// append + prefill entry when it runs as separate launches.
__global__ void __launch_bounds__(256) copy_lengths_kernel(const int32_t* seq_lens, int64_t* out, int B) {
  pdl_wait();
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < B; b += gridDim.x * blockDim.x) out[b] = seq_lens[b];
}

int launch_copy_lengths(const int32_t* seq_lens, int64_t* out, int B, cudaStream_t stream) {
  if (B <= 0 || out == nullptr) return B2PA_OK;
  const cudaError_t e = launch_pdl(copy_lengths_kernel, dim3((unsigned)((B + 255) / 256)), dim3(256), 0, stream,
                                   seq_lens, out, B);
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "copy_lengths launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

static bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

int launch_kv_append(const AppendArgs& a, cudaStream_t stream) {
  if (a.B == 0 || a.T == 0) return B2PA_OK;
  const int es = dtype_size(a.dtype);
  const int row_bytes = a.D * es;
  // Widest word that every source row start, destination row start and the
  // row length allow.  Destination rows start at multiples of row_bytes.
  int vb = 16;
  auto ok = [&](int w) {
    if (row_bytes % w) return false;
    if (!aligned(a.k_new, w) || !aligned(a.v_new, w) || !aligned(a.k_pool, w) || !aligned(a.v_pool, w)) return false;
    if (a.sk[3] != 1 || a.sv[3] != 1) return false;
    for (int i = 0; i < 3; ++i)
      if ((a.sk[i] * es) % w || (a.sv[i] * es) % w) return false;
    return true;
  };
  while (vb > es && !ok(vb)) vb >>= 1;
  dim3 grid(a.T, a.B);
  if (vb >= 4 && ok(vb)) {
    switch (vb) {
      case 16: launch_pdl(kv_append_kernel<16>, grid, dim3(128), 0, stream, a, es); break;
      case 8: launch_pdl(kv_append_kernel<8>, grid, dim3(128), 0, stream, a, es); break;
      default: launch_pdl(kv_append_kernel<4>, grid, dim3(128), 0, stream, a, es); break;
    }
  } else if (es == 2) {
    launch_pdl(kv_append_kernel_u16, grid, dim3(128), 0, stream, a);
  } else {
    // fp32 with a non-unit D stride: the rows cannot be moved as words.
    return set_error(B2PA_ERR_UNSUPPORTED, "kv_append: fp32 tensors need a unit D stride");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "kv_append launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

int launch_zero_blocks(const ZeroArgs& a, cudaStream_t stream) {
  if (a.n_ids == 0) return B2PA_OK;
  const int64_t block_bytes = (int64_t)a.H * a.block_size * a.D * dtype_size(a.dtype);
  const bool v16 = block_bytes % 16 == 0 && aligned(a.k_pool, 16) && aligned(a.v_pool, 16);
  if (v16)
    zero_blocks_kernel<16><<<a.n_ids, 256, 0, stream>>>(a, block_bytes);
  else
    zero_blocks_kernel<4><<<a.n_ids, 256, 0, stream>>>(a, block_bytes);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "zero_blocks launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

// One thread per (index, value) pair of a block-table patch.
__global__ void __launch_bounds__(256) patch_table_kernel(int32_t* table, int64_t n_cells, const int32_t* pairs,
                                                          int n_pairs, int32_t* status) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_pairs) return;
  const int32_t idx = pairs[2 * i];
  if (idx < 0 || (int64_t)idx >= n_cells) {
    set_status(status, B2PA_ERR_INVALID_ARGUMENT);
    return;
  }
  table[idx] = pairs[2 * i + 1];
}

int launch_patch_table(int32_t* table, int64_t n_cells, const int32_t* pairs, int n_pairs, int32_t* status,
                       cudaStream_t stream) {
  if (n_pairs == 0) return B2PA_OK;
  patch_table_kernel<<<(n_pairs + 255) / 256, 256, 0, stream>>>(table, n_cells, pairs, n_pairs, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "patch_table launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

}  // namespace b2pa
