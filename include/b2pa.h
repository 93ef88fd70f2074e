/*
 * b2pa.h -- C ABI of the B200 paged-attention backend (libb2pa.so).
 *
 * The library replaces three pieces of the reference serving stack
 * (jacobzhang22/efficient-inference-system):
 *
 *   - the per-token KV append/scatter into a layer's block pool
 *       src/cache/paged_kv.py:102-120 (PagedKVCacheState.append)
 *       src/cache/paged_kv.py:151-172 (BatchedPagedKVCache.append_batch)
 *   - the single-query paged decode attention launcher + kernel
 *       src/kernels/triton_paged_attention.py:10-85, 179-217
 *   - the chunked-prefill paged attention launcher + kernel
 *       src/kernels/triton_paged_attention.py:88-176, 220-258
 *
 * Data layout (unchanged from the reference, src/cache/paged_kv.py:54-62):
 *   k_pool, v_pool : [num_blocks, H, block_size, D], contiguous, dtype of q
 *   page_table     : int32 [B, max_pages], -1 padded (paged_kv.py:174-193)
 *   seq_lens       : int32 [B], length of each sequence AFTER the append
 *   cur_lens       : int32 [B], tokens added by this forward (attention.py:56-62)
 *   q, out         : [B, H, T, D] with arbitrary B/H/T strides, unit D stride
 *
 * Attention semantics (src/kernels/reference_paged_attention.py:31-57):
 *   query row t of sequence b sits at absolute position
 *       pos = seq_lens[b] - cur_lens[b] + t
 *   and sees keys 0 .. min(seq_lens[b], pos + 1) - 1.  Rows that see no key
 *   produce zeros.  out = softmax(q.K^T * scale) . V, accumulated in fp32,
 *   stored in the dtype of q.
 *
 * Conventions:
 *   - every entry point returns 0 (B2PA_OK) or a negative b2pa_status; no C++
 *     exception crosses the ABI.  b2pa_last_error_string() describes the most
 *     recent failure of the calling thread.
 *   - all pointers except `strides` arrays are DEVICE pointers owned by the
 *     caller; the library borrows them for the duration of the (asynchronous)
 *     call on `stream` (a cudaStream_t, NULL = legacy default stream).
 *   - the library never allocates device memory.  Scratch space is passed in
 *     as `workspace` (size from the matching *_workspace_size function).
 *   - `status` (nullable) is a device int32 that kernels set (first error
 *     wins) when they detect a fault they survived: an out-of-range block id
 *     or a bounded wait that gave up.  Read it with b2pa_status_read().
 *   - pool pointers are re-read on every call: the reference pool grows with
 *     torch.cat (paged_kv.py:64-69), which moves the tensors.
 */
#ifndef B2PA_H_
#define B2PA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2PA_ABI_VERSION 1

#if defined(__GNUC__)
#define B2PA_API __attribute__((visibility("default")))
#else
#define B2PA_API
#endif

typedef enum b2pa_dtype {
  B2PA_DTYPE_F32 = 0,
  B2PA_DTYPE_BF16 = 1,
  B2PA_DTYPE_F16 = 2
} b2pa_dtype;

typedef enum b2pa_status {
  B2PA_OK = 0,
  B2PA_ERR_INVALID_ARGUMENT = -1,  /* null pointer, negative size, bad stride */
  B2PA_ERR_UNSUPPORTED = -2,       /* dtype / head_dim / block_size not built */
  B2PA_ERR_BAD_BLOCK_ID = -3,      /* (device) page-table entry >= num_blocks */
  B2PA_ERR_WORKSPACE = -4,         /* workspace missing or too small */
  B2PA_ERR_CUDA = -5,              /* a CUDA runtime call failed */
  B2PA_ERR_DEVICE_TIMEOUT = -6     /* (device) a bounded wait gave up */
} b2pa_status;

/* ABI version of the loaded library (B2PA_ABI_VERSION at build time). */
B2PA_API int b2pa_abi_version(void);

/* Description of the calling thread's most recent error ("" if none). */
B2PA_API const char* b2pa_last_error_string(void);

/* Copies the device status word to *host_status (synchronises `stream`). */
B2PA_API int b2pa_status_read(const int32_t* status, int32_t* host_status, void* stream);

/* Clears the device status word (asynchronous on `stream`). */
B2PA_API int b2pa_status_clear(int32_t* status, void* stream);

/*
 * KV append / scatter.  Replaces the slice copies of
 * PagedKVCacheState.append (src/cache/paged_kv.py:109-120) for a whole batch
 * (BatchedPagedKVCache.append_batch, paged_kv.py:151-172) in one launch.
 *
 * For each sequence b and t < min(lengths[b], T):
 *   pos = start_pos[b] + t
 *   blk = page_table[b * pt_stride + pos / block_size]
 *   k_pool[blk, h, pos % block_size, :] = k_new[b, h, t, :]   (all h)
 *   v_pool[...]                          = v_new[b, h, t, :]
 * Block ids must already be allocated by the caller's host allocator in the
 * reference order (paged_kv.py:110-113); this kernel only copies, bit-exact.
 * new_k_strides / new_v_strides / pool_strides are element strides of the
 * [B,H,T,D] and [num_blocks,H,block_size,D] tensors.
 */
B2PA_API int b2pa_kv_append(const void* k_new, const int64_t new_k_strides[4],
                   const void* v_new, const int64_t new_v_strides[4],
                   void* k_pool, void* v_pool, const int64_t pool_strides[4],
                   int64_t num_blocks,
                   const int32_t* page_table, int64_t pt_stride, int max_pages,
                   const int32_t* start_pos, const int32_t* lengths,
                   int B, int H, int T, int D, int block_size, int dtype,
                   int32_t* status, void* stream);

/*
 * Workspace bytes b2pa_paged_decode needs for this problem size.  Replaces
 * nothing in the reference (the Triton decode kernel runs one program per
 * (seq, head) with no split, triton_paged_attention.py:189); the split-K
 * partials of this backend live here.  With at least 3 head-group streams
 * (B * H / heads per group) per SM of the current device, the size depends on
 * that device's SM count, not on max_pages: query it with the device current
 * that will run the call (a call given less is refused with
 * B2PA_ERR_WORKSPACE).
 */
B2PA_API size_t b2pa_paged_decode_workspace_size(int B, int H, int D, int max_pages,
                                        int block_size, int dtype);

/*
 * Single-query paged decode attention (T == 1).  Replaces
 * paged_attention_decode_triton, src/kernels/triton_paged_attention.py:179-217.
 * q_strides / out_strides: element strides of [B,H,1,D] (D stride must be 1).
 */
B2PA_API int b2pa_paged_decode(const void* q, const int64_t q_strides[4],
                      const void* k_pool, const void* v_pool,
                      const int64_t pool_strides[4], int64_t num_blocks,
                      const int32_t* page_table, int64_t pt_stride, int max_pages,
                      const int32_t* seq_lens, const int32_t* cur_lens,
                      void* out, const int64_t out_strides[4],
                      int B, int H, int D, int block_size, float scale, int dtype,
                      void* workspace, size_t workspace_bytes,
                      int32_t* status, void* stream);

/*
 * Decode with the step's KV append fused into the same launch.  Replaces the
 * pair CausalSelfAttention.forward makes for a decode step
 * (src/model/attention.py:56-62): BatchedPagedKVCache.append_batch with
 * T == 1 (src/cache/paged_kv.py:151-172, as b2pa_kv_append) followed by
 * paged_attention_decode_triton (src/kernels/triton_paged_attention.py:179-217,
 * as b2pa_paged_decode).  For each b with lengths[b] > 0, k_new[b,:,0,:] and
 * v_new[b,:,0,:] are written to pool position start_pos[b] (block
 * page_table[b, start_pos[b] / block_size]), and the attention of b sees
 * them: seq_lens are the lengths after the append, as for b2pa_paged_decode,
 * so start_pos[b] must be seq_lens[b] - 1 (rows where it is not are skipped
 * and B2PA_ERR_INVALID_ARGUMENT is set in the status word; a block id out of
 * range sets B2PA_ERR_BAD_BLOCK_ID).  The host allocator must already have
 * assigned the block.  seq_lens_out
 * (may be NULL) receives seq_lens as int64, the value append_batch returns.
 * k_new / v_new: [B,H,1,D] element strides, unit D stride, rows 4-byte
 * aligned.  Same workspace as b2pa_paged_decode.  Pool bytes and outputs are
 * identical to b2pa_kv_append followed by b2pa_paged_decode.
 */
B2PA_API int b2pa_paged_decode_append(const void* q, const int64_t q_strides[4],
                      const void* k_new, const int64_t new_k_strides[4],
                      const void* v_new, const int64_t new_v_strides[4],
                      void* k_pool, void* v_pool,
                      const int64_t pool_strides[4], int64_t num_blocks,
                      const int32_t* page_table, int64_t pt_stride, int max_pages,
                      const int32_t* seq_lens, const int32_t* cur_lens,
                      const int32_t* start_pos, const int32_t* lengths,
                      int64_t* seq_lens_out,
                      void* out, const int64_t out_strides[4],
                      int B, int H, int D, int block_size, float scale, int dtype,
                      void* workspace, size_t workspace_bytes,
                      int32_t* status, void* stream);

/*
 * Decode without a caller workspace.  No counterpart in the reference: this
 * entry point exists for callers that cannot allocate device memory (a host
 * callback or real-time thread that must not block on the allocator, a
 * plugin whose host framework owns all device memory, a process whose
 * footprint is fixed at start-up).  Same arguments and results as
 * b2pa_paged_decode without `workspace`; the scratch lives in a fixed array
 * of B2PA_NOALLOC_SCRATCH_BYTES inside the library, held on every GPU that
 * loads it until exit.  Problems whose b2pa_paged_decode_workspace_size()
 * exceeds that return B2PA_ERR_WORKSPACE.  All calls on a device share the
 * array: calls that may overlap on the GPU (unordered streams) race.  The
 * first call in each CUDA context looks the array up (cudaGetSymbolAddress),
 * so make it before any stream capture: a first call on a capturing stream
 * returns B2PA_ERR_UNSUPPORTED.  A context created anew on the device (after
 * cudaDeviceReset) looks the array up again.  Allocates nothing.
 */
#define B2PA_NOALLOC_SCRATCH_BYTES (32u << 20)
B2PA_API int b2pa_paged_decode_noalloc(const void* q, const int64_t q_strides[4],
                      const void* k_pool, const void* v_pool,
                      const int64_t pool_strides[4], int64_t num_blocks,
                      const int32_t* page_table, int64_t pt_stride, int max_pages,
                      const int32_t* seq_lens, const int32_t* cur_lens,
                      void* out, const int64_t out_strides[4],
                      int B, int H, int D, int block_size, float scale, int dtype,
                      int32_t* status, void* stream);

/*
 * Workspace bytes b2pa_paged_prefill needs (0 for the paths that need none).
 * bf16/fp16, and fp32 with head_dim 128: the split-K partials when the key
 * range is split (small batches).  fp32 with head_dim 64 (tensor cores on
 * fp16 hi/lo splits of the operands): also the split copies of the pages
 * the call may read -- B * max_pages * H * block_size * D * 8 bytes, the
 * size of those fp32 K and V pages -- and a small slot table.
 */
B2PA_API size_t b2pa_paged_prefill_workspace_size(int B, int H, int T, int D, int max_pages,
                                         int block_size, int dtype);

/*
 * Chunked-prefill paged attention (any T >= 1, padded rows included).
 * Replaces paged_attention_prefill_triton,
 * src/kernels/triton_paged_attention.py:220-258.  fp32 results match fp32
 * arithmetic to the fp32 tolerance on every path; with head_dim 64 the call
 * runs on the tensor cores unless an input has magnitude >= 2^15 or is not
 * finite, in which case a CUDA-core kernel recomputes it (same results,
 * slower).
 */
B2PA_API int b2pa_paged_prefill(const void* q, const int64_t q_strides[4],
                       const void* k_pool, const void* v_pool,
                       const int64_t pool_strides[4], int64_t num_blocks,
                       const int32_t* page_table, int64_t pt_stride, int max_pages,
                       const int32_t* seq_lens, const int32_t* cur_lens,
                       void* out, const int64_t out_strides[4],
                       int B, int H, int T, int D, int block_size, float scale,
                       int dtype, void* workspace, size_t workspace_bytes,
                       int32_t* status, void* stream);

/*
 * Chunked prefill with the chunk's KV append in the same call.  Replaces the
 * pair CausalSelfAttention.forward makes per layer for a prompt chunk
 * (src/model/attention.py:56-62): BatchedPagedKVCache.append_batch
 * (src/cache/paged_kv.py:151-172, as b2pa_kv_append) followed by
 * paged_attention_prefill_triton (src/kernels/triton_paged_attention.py:
 * 220-258, as b2pa_paged_prefill).  For each b, rows t < min(lengths[b], T)
 * of k_new / v_new ([B,H,T,D] element strides, unit D stride) go to pool
 * positions start_pos[b] + t, which must end at seq_lens[b] (the lengths
 * after the append; where the append is fused, see below, a sequence whose
 * rows do not is skipped and B2PA_ERR_INVALID_ARGUMENT set in the status
 * word); the attention of the chunk sees them.
 * seq_lens_out (may be NULL) receives seq_lens as int64, the value
 * append_batch returns.  For fp32 pools with head_dim 64 the append happens
 * inside the launch that copies the pages for the tensor cores; otherwise
 * the append kernel runs first.  Same workspace as b2pa_paged_prefill.  For
 * inputs that meet the contract above (start_pos[b] + min(lengths[b], T) ==
 * seq_lens[b], every page a row lands on present in the table) pool bytes and
 * outputs are identical to b2pa_kv_append followed by b2pa_paged_prefill.
 * Inputs that break it are handled differently by the two paths: the fused
 * fp32 path skips the offending rows and sets the status word, the others
 * append them as b2pa_kv_append would.
 */
B2PA_API int b2pa_paged_prefill_append(const void* q, const int64_t q_strides[4],
                       const void* k_new, const int64_t new_k_strides[4],
                       const void* v_new, const int64_t new_v_strides[4],
                       void* k_pool, void* v_pool,
                       const int64_t pool_strides[4], int64_t num_blocks,
                       const int32_t* page_table, int64_t pt_stride, int max_pages,
                       const int32_t* seq_lens, const int32_t* cur_lens,
                       const int32_t* start_pos, const int32_t* lengths,
                       int64_t* seq_lens_out,
                       void* out, const int64_t out_strides[4],
                       int B, int H, int T, int D, int block_size, float scale, int dtype,
                       void* workspace, size_t workspace_bytes,
                       int32_t* status, void* stream);

/*
 * Zeroes whole blocks of both pools in one launch.  Replaces the per-block
 * k_blocks[id].zero_() / v_blocks[id].zero_() pair of
 * LayerBlockPool.release_block, src/cache/paged_kv.py:80-85.
 */
B2PA_API int b2pa_zero_blocks(void* k_pool, void* v_pool, const int64_t pool_strides[4],
                     int64_t num_blocks, const int32_t* block_ids, int n_ids,
                     int H, int D, int block_size, int dtype,
                     int32_t* status, void* stream);

/*
 * Writes table[pairs[2i]] = pairs[2i+1] for i < n_pairs: an in-place update
 * of a device-resident int32 block table (or any int32 array of n_cells
 * entries).  No reference counterpart: the reference rebuilds the whole
 * [B, max_pages] table from Python lists and copies it to the device on every
 * call (BatchedPagedKVCache.page_table_tensor, src/cache/paged_kv.py:174-193);
 * this lets the caller keep the table resident and send only the cells that
 * changed.  An index outside [0, n_cells) is skipped and recorded as
 * B2PA_ERR_INVALID_ARGUMENT in *status.
 */
B2PA_API int b2pa_patch_table(int32_t* table, int64_t n_cells, const int32_t* pairs, int n_pairs,
                     int32_t* status, void* stream);

/*
 * Failure-path self-test; no reference counterpart (the reference has no
 * failure detection).  Launches one warp that waits, through the bounded
 * wait every b2pa kernel uses, on an mbarrier that nothing arrives at: after
 * about one second the wait gives up, B2PA_ERR_DEVICE_TIMEOUT is recorded in
 * *status, *done (device int32) is set to 2 and the kernel returns, leaving
 * the CUDA context usable.  Lets a test check the give-up path without
 * faulting or hanging the GPU.
 */
B2PA_API int b2pa_selftest_wait_timeout(int32_t* status, int32_t* done, void* stream);

/*
 * The non-attention operations of a decode step, fp32, for M <= 16 rows (the
 * batch's new tokens).  In the reference they are torch modules of the
 * model: nn.LayerNorm, nn.Linear and nn.GELU of TransformerBlock
 * (src/model/transformer.py:10-18,27-34), the q/k/v and output projections of
 * CausalSelfAttention (src/model/attention.py:46-48,64), the embeddings, final
 * LayerNorm and lm_head of TinyTransformerLM (src/model/transformer.py:
 * 150,179-180) and the greedy torch.argmax of generation
 * (src/inference/generate_with_cache.py:204).  With M rows every product is
 * a matrix-vector product bound by reading the weights, so each call reads
 * its weight matrix once, with the row-wise work fused around it.
 *
 * b2pa_rows_linear: for each row m < M of x ([M, K], row stride
 * x_row_stride), xn = LayerNorm(x[m]) with ln_weight / ln_bias / ln_eps when
 * ln_weight is not NULL (ln_bias may be NULL), else x[m]; then
 * r[n] = xn . weight[n, :] + bias[n] (weight [N, K] row-major; bias may be
 * NULL), GELU (erf form) when activation == 1; y[m, n] = r[n], or
 * y[m, n] += r[n] when accumulate (a residual add).  y must not overlap x.
 * K a multiple of 4, M * K <= 32768, x / weight / LayerNorm vectors 16-byte
 * aligned with 16-byte row strides.
 */
B2PA_API int b2pa_rows_linear(const float* x, int64_t x_row_stride, int M, int K,
                              const float* ln_weight, const float* ln_bias, float ln_eps,
                              const float* weight, const float* bias, int N, int activation,
                              float* y, int64_t y_row_stride, int accumulate,
                              int32_t* status, void* stream);

/*
 * x[m, :] = token_table[token_ids[m], :] + position_table[positions[m], :]
 * for m < M (int64 ids on the device; tables [vocab, K] and
 * [max_positions, K], K a multiple of 4).  An id outside its table writes a
 * zero row and sets B2PA_ERR_INVALID_ARGUMENT in *status.
 */
B2PA_API int b2pa_rows_embed(const int64_t* token_ids, const int64_t* positions, int M,
                             const float* token_table, int64_t vocab,
                             const float* position_table, int64_t max_positions, int K,
                             float* x, int64_t x_row_stride, int32_t* status, void* stream);

/* out[m] = the first index of the largest of x[m, 0:N] (int64), m < M. */
B2PA_API int b2pa_rows_argmax(const float* x, int64_t x_row_stride, int M, int N, int64_t* out,
                              int32_t* status, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* B2PA_H_ */
