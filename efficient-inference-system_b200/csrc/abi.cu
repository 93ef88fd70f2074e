// abi.cu -- extern "C" entry points of libb2pa.so (declared in b2pa.h).
//
// Each entry point validates its arguments on the host, maps them onto the
// launcher structs of kernels.h and enqueues the kernels on the caller's
// stream.  Nothing here allocates device memory or synchronises, except the
// explicit b2pa_status_read().  Errors come back as b2pa_status codes with a
// thread-local message; no C++ exception crosses the ABI.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "b2pa.h"
#include "kernels.h"

namespace b2pa {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

static int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

static constexpr int kMaxDevices = 64;

int device_sm_count() {
  static int cache[kMaxDevices] = {0};
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

int device_max_smem_optin() {
  static int cache[kMaxDevices] = {0};
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 227 * 1024;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cache[dev] = n > 0 ? n : 227 * 1024;
  }
  return cache[dev];
}

int set_max_dynamic_smem_cached(const void* func, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes already allowed
  const auto key = std::make_pair(func, current_device());
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return B2PA_OK;
  }
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "cudaFuncSetAttribute(%d bytes): %s", bytes, cudaGetErrorString(e));
  std::lock_guard<std::mutex> g(mu);
  int& v = done[key];
  if (bytes > v) v = bytes;
  return B2PA_OK;
}

int decode_occupancy_cached(const void* func, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t, int>, int> cache;
  const auto key = std::make_tuple(func, threads, smem, current_device());
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, threads, smem) != cudaSuccess) n = 0;
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n;
  return n;
}

// Split size: about one work item per resident CTA (148 SMs x 3 CTAs), so
// that a short call runs in about one wave, with pages per split kept
// between 4 and 64.  Measured on config[1] (64 sequences of 128-1024 tokens,
// fp32, 444 CTAs), decode call time by item target: 2048 -> 40.8 us,
// 1024 -> 39.2, 512 -> 38.7, 256 -> 43.0, no split -> 56.1: finer splits
// cost more in partials and merging than they gain in balance, coarser ones
// leave SMs idle behind the longest sequences.
static int choose_pages_per_split(int B, int HG, int max_pages) {
  const int64_t target_items = 512;
  const int64_t pairs = (int64_t)B * HG;
  int64_t splits = pairs > 0 ? (target_items + pairs - 1) / pairs : 1;
  if (splits < 1) splits = 1;
  int64_t P = (max_pages + splits - 1) / splits;
  if (P < 4) P = 4;
  if (P > 64) P = 64;
  return (int)P;
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

DecodePlan make_decode_plan(int B, int H, int D, int max_pages, int block_size, int dtype) {
  DecodePlan pl;
  const int hpb = block_size * D * dtype_size(dtype);
  int G = 1;
  for (int g : {4, 2}) {
    if (H % g == 0 && 2 * g * hpb <= 48 * 1024) {
      G = g;
      break;
    }
  }
  pl.G = G;
  pl.HG = H / G;
  pl.pages_per_split = choose_pages_per_split(B, pl.HG, max_pages);
  const int64_t splits = max_pages > 0 ? (max_pages + pl.pages_per_split - 1) / pl.pages_per_split : 1;
  pl.max_items = (int64_t)B * pl.HG * (splits > 0 ? splits : 1);
  // Contiguous split (each CTA streams an equal range of the flattened
  // (sequence, head group, page) units; a stream cut between CTAs leaves one
  // partial per piece) when there are at least as many streams as a typical
  // grid has CTAs (148 SMs x 3).  Then the item split has more than one item
  // per CTA and quantises into waves, while the ranges balance the SMs
  // exactly; with fewer streams the item split measured faster (the extra
  // pieces of the ranges cost more than they save).  Measured per decode
  // call (bf16, H=32, D=128 unless noted; short: L ~ U[128,1024], long:
  // U[1024,8192]; item -> contiguous split): 128 streams
  // (config[1], fp32, H=8, D=64) 33.6 -> 36.6 us; 128 long streams 224.7 ->
  // 228.5 us; 256 short streams 69.7 -> 75.5 us; 512 short streams 165.1 ->
  // 124.8 us; 512 / 1,024 / 2,048 / 4,096 long streams (config[4], 64 to
  // 512 sequences) 4.8 / 2.7 / 2.2 / 2.9 % faster.
  const int64_t max_ctas = (int64_t)device_sm_count() * kDecodeMaxCtasPerSm;
  const int64_t units = (int64_t)B * pl.HG * (max_pages > 0 ? max_pages : 1);
  pl.contig =
      (int64_t)B * pl.HG >= (int64_t)kDecodeContigStreamsPerSm * device_sm_count() && units <= INT32_MAX ? 1 : 0;
  if (pl.contig) pl.max_items = 2 * max_ctas;
  size_t off = 0;
  pl.off_item_off = off;
  off = align_up(off + 4ull * (B + 1), 256);
  pl.off_part_ml = off;
  off = align_up(off + 8ull * pl.max_items * G, 256);
  pl.off_part_acc = off;
  off = align_up(off + 4ull * pl.max_items * G * D, 256);
  pl.bytes = off;
  return pl;
}

bool prefill_uses_tensor_cores(int D, int block_size, int dtype, int64_t pool_rows) {
  return (dtype == B2PA_DTYPE_BF16 || dtype == B2PA_DTYPE_F16) && (D == 64 || D == 128) &&
         (block_size == 8 || block_size == 16 || block_size == 32) && pool_rows <= ((int64_t)1 << 31);
}

// Split the key range of the tensor-core prefill (query tiles of 128 rows)
// when the (query tile, head, sequence) CTAs alone would leave SMs idle: the
// split CTAs fill one wave of `slots` resident CTAs (148 SMs, one CTA each),
// at least 2 key tiles each.  Measured on config[2]: a second wave, or a
// second resident CTA per SM (a 99 KB, one-softmax-group variant sized for
// two per SM was built and ran 19.4 -> 31.7 us), costs more than the shorter
// key walks save.  Sets kt_per_split / nsplit_max and
// the partials' workspace offsets; returns the partials' bytes.
static size_t tc_key_split(PrefillPlan& pl, int B, int H, int T, int D, int64_t ktmax, int64_t slots,
                           int64_t kt_cap) {
  if (B <= 0 || T <= 0 || ktmax <= 2) return 0;
  const int64_t ctas = (int64_t)B * H * ((T + 127) / 128);
  int64_t splits = slots / ctas;
  // Each split keeps at least 8 key tiles: a split saves ~0.4 us per tile it
  // takes off the longest CTA and costs the combine pass (~3 us, measured: a
  // 4-tile range split in two ran 14.3 -> 18.4 us).
  if (splits > ktmax / 8) splits = ktmax / 8;
  // A CTA stages the block ids of its key range in shared memory: at most
  // kt_cap key tiles per CTA.
  const int64_t min_splits = (ktmax + kt_cap - 1) / kt_cap;
  if (splits < min_splits) splits = min_splits;
  if (splits > ktmax) splits = ktmax;
  if (splits <= 1) return 0;
  int64_t kt = (ktmax + splits - 1) / splits;
  if (kt < 2) kt = 2;
  const int64_t ns = (ktmax + kt - 1) / kt;
  if (ns <= 1) return 0;
  pl.kt_per_split = (int)kt;
  pl.nsplit_max = (int)ns;
  const size_t nslots = (size_t)B * H * T * ns;
  pl.off_part_ml = 0;
  pl.off_part_o = align_up(8 * nslots, 256);
  return align_up(pl.off_part_o + 4 * nslots * D, 256);
}

static bool prefill_f32_split_tc(int D, int block_size, int64_t split_rows) {
  return D == 64 && (block_size == 8 || block_size == 16 || block_size == 32) && split_rows > 0 &&
         split_rows <= ((int64_t)1 << 31);
}

static PrefillPlan empty_prefill_plan(int64_t ktmax) {
  PrefillPlan pl;
  pl.bm = 128;
  pl.kt_per_split = (int)(ktmax > 0 ? ktmax : 1);
  pl.nsplit_max = 1;
  pl.split_tc = 0;
  pl.off_part_ml = pl.off_part_o = pl.off_split_k = pl.off_split_v = pl.off_slots = pl.off_flag = 0;
  pl.bytes = 0;
  return pl;
}

PrefillPlan make_prefill_plan_f32_tiled(int B, int H, int T, int D, int max_pages, int block_size) {
  // fp32 register-tiled kernel (64-row query tiles): a CTA takes at most
  // kFp32KtCap key tiles, so the longest causal rows do not set the length
  // of the whole launch; the splits are merged by the combine kernel.
  constexpr int64_t kFp32KtCap = 8;
  const int64_t ktmax = ((int64_t)max_pages * block_size + 63) / 64;
  PrefillPlan pl = empty_prefill_plan(ktmax);
  pl.bm = 64;
  if (B <= 0 || T <= 0 || ktmax <= kFp32KtCap) return pl;
  const int64_t ns = (ktmax + kFp32KtCap - 1) / kFp32KtCap;
  const int64_t kt = (ktmax + ns - 1) / ns;
  pl.kt_per_split = (int)kt;
  pl.nsplit_max = (int)((ktmax + kt - 1) / kt);
  const size_t slots = (size_t)B * H * T * pl.nsplit_max;
  pl.off_part_ml = 0;
  pl.off_part_o = align_up(8 * slots, 256);
  pl.bytes = align_up(pl.off_part_o + 4 * slots * D, 256);
  return pl;
}

PrefillPlan make_prefill_plan(int B, int H, int T, int D, int max_pages, int block_size, int dtype) {
  const int64_t ktmax = ((int64_t)max_pages * block_size + 63) / 64;
  PrefillPlan pl = empty_prefill_plan(ktmax);
  if (dtype == B2PA_DTYPE_F32 && B > 0 && T > 0 &&
      prefill_f32_split_tc(D, block_size, (int64_t)B * max_pages * H * block_size)) {
    // fp32, head_dim 64: the tensor-core kernel on fp16 hi/lo copies of the
    // pages (B * max_pages slots of H pages, K and V, 2 * D halves per row),
    // after the partials of its key-range split; then the range flag.
    pl.split_tc = 1;
    const size_t part = tc_key_split(pl, B, H, T, D, ktmax, 148, 1024);
    const size_t slot_bytes = (size_t)H * block_size * 2 * D * 2;
    const size_t nslots = (size_t)B * max_pages;
    pl.off_split_k = align_up(part, 256);
    pl.off_split_v = align_up(pl.off_split_k + nslots * slot_bytes, 256);
    pl.off_slots = align_up(pl.off_split_v + nslots * slot_bytes, 256);
    pl.off_flag = align_up(pl.off_slots + 4 * nslots, 256);
    pl.bytes = pl.off_flag + 256;
    return pl;
  }
  if (dtype == B2PA_DTYPE_F32 && (D == 64 || D == 128))
    return make_prefill_plan_f32_tiled(B, H, T, D, max_pages, block_size);
  if (!prefill_uses_tensor_cores(D, block_size, dtype, 0)) return pl;
  pl.bytes = tc_key_split(pl, B, H, T, D, ktmax, 148, 1024);
  return pl;
}

}  // namespace b2pa

using namespace b2pa;

namespace {

bool aligned_to(const void* p, size_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; }

// Shared validation of the attention entry points.  Returns B2PA_OK or an
// error code with the message set.
int validate_attention(const char* fn, const void* q, const int64_t* qs, const void* k_pool, const void* v_pool,
                       const int64_t* ps, int64_t num_blocks, const int32_t* page_table, int64_t pt_stride,
                       int max_pages, const int32_t* seq_lens, const int32_t* cur_lens, void* out,
                       const int64_t* os, int B, int H, int T, int D, int block_size, int dtype) {
  if (B < 0 || H <= 0 || T < 0 || D <= 0 || block_size <= 0 || max_pages < 0 || num_blocks < 0)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "%s: bad sizes B=%d H=%d T=%d D=%d block_size=%d max_pages=%d", fn, B,
                     H, T, D, block_size, max_pages);
  if (dtype_size(dtype) == 0) return set_error(B2PA_ERR_UNSUPPORTED, "%s: unknown dtype %d", fn, dtype);
  if (!head_dim_supported(D)) return set_error(B2PA_ERR_UNSUPPORTED, "%s: head_dim %d not built", fn, D);
  if (!block_size_supported(block_size))
    return set_error(B2PA_ERR_UNSUPPORTED, "%s: block_size %d not built", fn, block_size);
  if (B == 0 || T == 0) return B2PA_OK;
  if (!q || !k_pool || !v_pool || !seq_lens || !cur_lens || !out || !qs || !ps || !os)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (max_pages > 0 && !page_table) return set_error(B2PA_ERR_INVALID_ARGUMENT, "%s: null page_table", fn);
  if (max_pages > 0 && pt_stride < max_pages)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "%s: page-table row stride %lld < max_pages %d", fn,
                     (long long)pt_stride, max_pages);
  const int64_t es = dtype_size(dtype);
  if (ps[3] != 1 || ps[2] != D || ps[1] != (int64_t)block_size * D || ps[0] != (int64_t)H * block_size * D)
    return set_error(B2PA_ERR_UNSUPPORTED, "%s: pools must be contiguous [num_blocks, H, block_size, D]", fn);
  if (!aligned_to(k_pool, 16) || !aligned_to(v_pool, 16))
    return set_error(B2PA_ERR_UNSUPPORTED, "%s: pool base pointers must be 16-byte aligned", fn);
  if (qs[3] != 1 || os[3] != 1) return set_error(B2PA_ERR_UNSUPPORTED, "%s: q/out need a unit D stride", fn);
  // Rows of q and out are moved as 16-byte words (or narrower for D*es < 16).
  const int64_t row_align = (D * es) >= 16 ? 16 : D * es;
  if (!aligned_to(q, row_align) || !aligned_to(out, row_align))
    return set_error(B2PA_ERR_UNSUPPORTED, "%s: q/out must be %lld-byte aligned", fn, (long long)row_align);
  for (int i = 0; i < 3; ++i)
    if ((qs[i] * es) % row_align || (os[i] * es) % row_align)
      return set_error(B2PA_ERR_UNSUPPORTED, "%s: q/out strides must keep rows %lld-byte aligned", fn,
                       (long long)row_align);
  return B2PA_OK;
}

AttnArgs make_attn_args(const void* q, const int64_t* qs, const void* k_pool, const void* v_pool, int64_t num_blocks,
                        const int32_t* page_table, int64_t pt_stride, int max_pages, const int32_t* seq_lens,
                        const int32_t* cur_lens, void* out, const int64_t* os, int B, int H, int T, int D,
                        int block_size, float scale, int dtype, void* workspace, size_t workspace_bytes,
                        int32_t* status) {
  AttnArgs a = {};
  a.q = q;
  for (int i = 0; i < 4; ++i) {
    a.sq[i] = qs[i];
    a.so[i] = os[i];
  }
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.page_table = page_table;
  a.pt_stride = pt_stride;
  a.max_pages = max_pages;
  a.seq_lens = seq_lens;
  a.cur_lens = cur_lens;
  a.out = out;
  a.B = B;
  a.H = H;
  a.T = T;
  a.D = D;
  a.block_size = block_size;
  a.dtype = dtype;
  a.scale = scale;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  a.status = status;
  a.k_new = a.v_new = nullptr;
  a.skn[0] = a.skn[1] = a.skn[2] = a.svn[0] = a.svn[1] = a.svn[2] = 0;
  a.app_start = a.app_len = nullptr;
  a.app_vb = 0;
  a.seq_out = nullptr;
  return a;
}

}  // namespace

extern "C" {

int b2pa_abi_version(void) { return B2PA_ABI_VERSION; }

const char* b2pa_last_error_string(void) { return g_last_error.c_str(); }

int b2pa_status_read(const int32_t* status, int32_t* host_status, void* stream) {
  if (!status || !host_status) return set_error(B2PA_ERR_INVALID_ARGUMENT, "status_read: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(host_status, status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "status_read: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

int b2pa_status_clear(int32_t* status, void* stream) {
  if (!status) return set_error(B2PA_ERR_INVALID_ARGUMENT, "status_clear: null pointer");
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int32_t), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "status_clear: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

int b2pa_kv_append(const void* k_new, const int64_t new_k_strides[4], const void* v_new,
                   const int64_t new_v_strides[4], void* k_pool, void* v_pool, const int64_t pool_strides[4],
                   int64_t num_blocks, const int32_t* page_table, int64_t pt_stride, int max_pages,
                   const int32_t* start_pos, const int32_t* lengths, int B, int H, int T, int D, int block_size,
                   int dtype, int32_t* status, void* stream) {
  if (B < 0 || H <= 0 || T < 0 || D <= 0 || block_size <= 0 || max_pages < 0 || num_blocks < 0)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "kv_append: bad sizes B=%d H=%d T=%d D=%d block_size=%d", B, H, T, D,
                     block_size);
  if (dtype_size(dtype) == 0) return set_error(B2PA_ERR_UNSUPPORTED, "kv_append: unknown dtype %d", dtype);
  if (B == 0 || T == 0) return B2PA_OK;
  if (!k_new || !v_new || !k_pool || !v_pool || !new_k_strides || !new_v_strides || !pool_strides || !start_pos ||
      !lengths)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "kv_append: null pointer argument");
  if (max_pages > 0 && (!page_table || pt_stride < max_pages))
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "kv_append: bad page table");
  const int64_t* ps = pool_strides;
  if (ps[3] != 1 || ps[2] != D || ps[1] != (int64_t)block_size * D || ps[0] != (int64_t)H * block_size * D)
    return set_error(B2PA_ERR_UNSUPPORTED, "kv_append: pools must be contiguous [num_blocks, H, block_size, D]");
  AppendArgs a;
  a.k_new = k_new;
  a.v_new = v_new;
  for (int i = 0; i < 4; ++i) {
    a.sk[i] = new_k_strides[i];
    a.sv[i] = new_v_strides[i];
  }
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.page_table = page_table;
  a.pt_stride = pt_stride;
  a.max_pages = max_pages;
  a.start_pos = start_pos;
  a.lengths = lengths;
  a.B = B;
  a.H = H;
  a.T = T;
  a.D = D;
  a.block_size = block_size;
  a.dtype = dtype;
  a.status = status;
  return launch_kv_append(a, static_cast<cudaStream_t>(stream));
}

size_t b2pa_paged_decode_workspace_size(int B, int H, int D, int max_pages, int block_size, int dtype) {
  if (B <= 0 || H <= 0 || D <= 0 || max_pages < 0 || block_size <= 0 || dtype_size(dtype) == 0) return 0;
  return make_decode_plan(B, H, D, max_pages, block_size, dtype).bytes;
}

int b2pa_paged_decode(const void* q, const int64_t q_strides[4], const void* k_pool, const void* v_pool,
                      const int64_t pool_strides[4], int64_t num_blocks, const int32_t* page_table,
                      int64_t pt_stride, int max_pages, const int32_t* seq_lens, const int32_t* cur_lens, void* out,
                      const int64_t out_strides[4], int B, int H, int D, int block_size, float scale, int dtype,
                      void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  int rc = validate_attention("paged_decode", q, q_strides, k_pool, v_pool, pool_strides, num_blocks, page_table,
                              pt_stride, max_pages, seq_lens, cur_lens, out, out_strides, B, H, 1, D, block_size,
                              dtype);
  if (rc != B2PA_OK || B == 0) return rc;
  const DecodePlan plan = make_decode_plan(B, H, D, max_pages, block_size, dtype);
  if (!workspace || workspace_bytes < plan.bytes)
    return set_error(B2PA_ERR_WORKSPACE, "paged_decode: workspace of %zu bytes, %zu needed", workspace_bytes,
                     plan.bytes);
  if (!aligned_to(workspace, 256)) return set_error(B2PA_ERR_WORKSPACE, "paged_decode: workspace must be 256-byte aligned");
  if (plan.max_items > INT32_MAX)
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode: %lld work items exceed the int32 plan", (long long)plan.max_items);
  AttnArgs a = make_attn_args(q, q_strides, k_pool, v_pool, num_blocks, page_table, pt_stride, max_pages, seq_lens,
                              cur_lens, out, out_strides, B, H, 1, D, block_size, scale, dtype, workspace,
                              workspace_bytes, status);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case B2PA_DTYPE_F32: return launch_paged_decode_f32(a, plan, s);
    case B2PA_DTYPE_BF16: return launch_paged_decode_bf16(a, plan, s);
    default: return launch_paged_decode_f16(a, plan, s);
  }
}

int b2pa_paged_decode_append(const void* q, const int64_t q_strides[4], const void* k_new,
                             const int64_t new_k_strides[4], const void* v_new, const int64_t new_v_strides[4],
                             void* k_pool, void* v_pool, const int64_t pool_strides[4], int64_t num_blocks,
                             const int32_t* page_table, int64_t pt_stride, int max_pages, const int32_t* seq_lens,
                             const int32_t* cur_lens, const int32_t* start_pos, const int32_t* lengths,
                             int64_t* seq_lens_out, void* out, const int64_t out_strides[4], int B, int H, int D,
                             int block_size, float scale, int dtype, void* workspace, size_t workspace_bytes,
                             int32_t* status, void* stream) {
  int rc = validate_attention("paged_decode_append", q, q_strides, k_pool, v_pool, pool_strides, num_blocks,
                              page_table, pt_stride, max_pages, seq_lens, cur_lens, out, out_strides, B, H, 1, D,
                              block_size, dtype);
  if (rc != B2PA_OK || B == 0) return rc;
  if (!k_new || !v_new || !new_k_strides || !new_v_strides || !start_pos || !lengths)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "paged_decode_append: null pointer argument");
  const int64_t* ps = pool_strides;
  if (ps[3] != 1 || ps[2] != D || ps[1] != (int64_t)block_size * D || ps[0] != (int64_t)H * block_size * D)
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode_append: pools must be contiguous [num_blocks, H, block_size, D]");
  if (new_k_strides[3] != 1 || new_v_strides[3] != 1)
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode_append: k_new/v_new need a unit head_dim stride");
  // Widest access (16, 8 or 4 bytes) that every source row start allows;
  // pool rows start at multiples of D * element size.
  const int es = dtype_size(dtype);
  int vb = 16;
  auto fits = [&](int w) {
    if ((D * es) % w || !aligned_to(k_new, w) || !aligned_to(v_new, w) || !aligned_to(k_pool, w) ||
        !aligned_to(v_pool, w))
      return false;
    for (int i = 0; i < 2; ++i)
      if ((new_k_strides[i] * es) % w || (new_v_strides[i] * es) % w) return false;
    return true;
  };
  while (vb >= 4 && !fits(vb)) vb >>= 1;
  if (vb < 4)
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode_append: k_new/v_new rows are not 4-byte aligned");
  const DecodePlan plan = make_decode_plan(B, H, D, max_pages, block_size, dtype);
  if (!workspace || workspace_bytes < plan.bytes)
    return set_error(B2PA_ERR_WORKSPACE, "paged_decode_append: workspace of %zu bytes, %zu needed", workspace_bytes,
                     plan.bytes);
  if (!aligned_to(workspace, 256))
    return set_error(B2PA_ERR_WORKSPACE, "paged_decode_append: workspace must be 256-byte aligned");
  if (plan.max_items > INT32_MAX)
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode_append: %lld work items exceed the int32 plan",
                     (long long)plan.max_items);
  AttnArgs a = make_attn_args(q, q_strides, k_pool, v_pool, num_blocks, page_table, pt_stride, max_pages, seq_lens,
                              cur_lens, out, out_strides, B, H, 1, D, block_size, scale, dtype, workspace,
                              workspace_bytes, status);
  a.k_new = k_new;
  a.v_new = v_new;
  a.skn[0] = new_k_strides[0];
  a.skn[1] = new_k_strides[1];
  a.svn[0] = new_v_strides[0];
  a.svn[1] = new_v_strides[1];
  a.app_start = start_pos;
  a.app_len = lengths;
  a.app_vb = vb;
  a.seq_out = seq_lens_out;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case B2PA_DTYPE_F32: return launch_paged_decode_f32(a, plan, s);
    case B2PA_DTYPE_BF16: return launch_paged_decode_bf16(a, plan, s);
    default: return launch_paged_decode_f16(a, plan, s);
  }
}

size_t b2pa_paged_prefill_workspace_size(int B, int H, int T, int D, int max_pages, int block_size, int dtype) {
  if (B <= 0 || H <= 0 || T <= 0 || D <= 0 || max_pages < 0 || block_size <= 0 || dtype_size(dtype) == 0) return 0;
  return make_prefill_plan(B, H, T, D, max_pages, block_size, dtype).bytes;
}

int b2pa_paged_prefill(const void* q, const int64_t q_strides[4], const void* k_pool, const void* v_pool,
                       const int64_t pool_strides[4], int64_t num_blocks, const int32_t* page_table,
                       int64_t pt_stride, int max_pages, const int32_t* seq_lens, const int32_t* cur_lens, void* out,
                       const int64_t out_strides[4], int B, int H, int T, int D, int block_size, float scale,
                       int dtype, void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  int rc = validate_attention("paged_prefill", q, q_strides, k_pool, v_pool, pool_strides, num_blocks, page_table,
                              pt_stride, max_pages, seq_lens, cur_lens, out, out_strides, B, H, T, D, block_size,
                              dtype);
  if (rc != B2PA_OK || B == 0 || T == 0) return rc;
  if (T > 65535 * 32) return set_error(B2PA_ERR_UNSUPPORTED, "paged_prefill: T=%d too large", T);
  AttnArgs a = make_attn_args(q, q_strides, k_pool, v_pool, num_blocks, page_table, pt_stride, max_pages, seq_lens,
                              cur_lens, out, out_strides, B, H, T, D, block_size, scale, dtype, workspace,
                              workspace_bytes, status);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case B2PA_DTYPE_F32: return launch_paged_prefill_f32(a, s);
    case B2PA_DTYPE_BF16: return launch_paged_prefill_bf16(a, s);
    default: return launch_paged_prefill_f16(a, s);
  }
}

int b2pa_paged_prefill_append(const void* q, const int64_t q_strides[4], const void* k_new,
                              const int64_t new_k_strides[4], const void* v_new, const int64_t new_v_strides[4],
                              void* k_pool, void* v_pool, const int64_t pool_strides[4], int64_t num_blocks,
                              const int32_t* page_table, int64_t pt_stride, int max_pages, const int32_t* seq_lens,
                              const int32_t* cur_lens, const int32_t* start_pos, const int32_t* lengths,
                              int64_t* seq_lens_out, void* out, const int64_t out_strides[4], int B, int H, int T,
                              int D, int block_size, float scale, int dtype, void* workspace, size_t workspace_bytes,
                              int32_t* status, void* stream) {
  int rc = validate_attention("paged_prefill_append", q, q_strides, k_pool, v_pool, pool_strides, num_blocks,
                              page_table, pt_stride, max_pages, seq_lens, cur_lens, out, out_strides, B, H, T, D,
                              block_size, dtype);
  if (rc != B2PA_OK || B == 0 || T == 0) return rc;
  if (T > 65535 * 32) return set_error(B2PA_ERR_UNSUPPORTED, "paged_prefill_append: T=%d too large", T);
  if (!k_new || !v_new || !new_k_strides || !new_v_strides || !start_pos || !lengths)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "paged_prefill_append: null pointer argument");
  if (new_k_strides[3] != 1 || new_v_strides[3] != 1)
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_prefill_append: k_new/v_new need a unit head_dim stride");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  AttnArgs a = make_attn_args(q, q_strides, k_pool, v_pool, num_blocks, page_table, pt_stride, max_pages, seq_lens,
                              cur_lens, out, out_strides, B, H, T, D, block_size, scale, dtype, workspace,
                              workspace_bytes, status);
  // The fp32 split path copies every page the call reads anyway: its pre-pass
  // takes the new rows from k_new / v_new (16-byte rows) and writes them into
  // the pool as well.  Every other path appends first, with the append kernel.
  const int es = dtype_size(dtype);
  bool rows16 = aligned_to(k_new, 16) && aligned_to(v_new, 16);
  for (int i = 0; i < 3; ++i) rows16 = rows16 && (new_k_strides[i] * es) % 16 == 0 && (new_v_strides[i] * es) % 16 == 0;
  if (dtype == B2PA_DTYPE_F32 && rows16 &&
      make_prefill_plan(B, H, T, D, max_pages, block_size, dtype).split_tc) {
    a.k_new = k_new;
    a.v_new = v_new;
    for (int i = 0; i < 3; ++i) {
      a.skn[i] = new_k_strides[i];
      a.svn[i] = new_v_strides[i];
    }
    a.app_start = start_pos;
    a.app_len = lengths;
    a.seq_out = seq_lens_out;
    return launch_paged_prefill_f32(a, s);
  }
  rc = b2pa_kv_append(k_new, new_k_strides, v_new, new_v_strides, k_pool, v_pool, pool_strides, num_blocks, page_table,
                      pt_stride, max_pages, start_pos, lengths, B, H, T, D, block_size, dtype, status, stream);
  if (rc != B2PA_OK) return rc;
  a.after_append = 1;
  switch (dtype) {
    case B2PA_DTYPE_F32: rc = launch_paged_prefill_f32(a, s); break;
    case B2PA_DTYPE_BF16: rc = launch_paged_prefill_bf16(a, s); break;
    default: rc = launch_paged_prefill_f16(a, s); break;
  }
  if (rc != B2PA_OK) return rc;
  return launch_copy_lengths(seq_lens, seq_lens_out, B, s);
}

int b2pa_zero_blocks(void* k_pool, void* v_pool, const int64_t pool_strides[4], int64_t num_blocks,
                     const int32_t* block_ids, int n_ids, int H, int D, int block_size, int dtype, int32_t* status,
                     void* stream) {
  if (n_ids < 0 || H <= 0 || D <= 0 || block_size <= 0 || num_blocks < 0)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "zero_blocks: bad sizes");
  if (dtype_size(dtype) == 0) return set_error(B2PA_ERR_UNSUPPORTED, "zero_blocks: unknown dtype %d", dtype);
  if (n_ids == 0) return B2PA_OK;
  if (!k_pool || !v_pool || !block_ids || !pool_strides)
    return set_error(B2PA_ERR_INVALID_ARGUMENT, "zero_blocks: null pointer argument");
  const int64_t* ps = pool_strides;
  if (ps[3] != 1 || ps[2] != D || ps[1] != (int64_t)block_size * D || ps[0] != (int64_t)H * block_size * D)
    return set_error(B2PA_ERR_UNSUPPORTED, "zero_blocks: pools must be contiguous");
  ZeroArgs a;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.block_ids = block_ids;
  a.n_ids = n_ids;
  a.H = H;
  a.D = D;
  a.block_size = block_size;
  a.dtype = dtype;
  a.status = status;
  return launch_zero_blocks(a, static_cast<cudaStream_t>(stream));
}

int b2pa_patch_table(int32_t* table, int64_t n_cells, const int32_t* pairs, int n_pairs, int32_t* status,
                     void* stream) {
  if (n_pairs < 0 || n_cells < 0) return set_error(B2PA_ERR_INVALID_ARGUMENT, "patch_table: bad sizes");
  if (n_pairs == 0) return B2PA_OK;
  if (!table || !pairs) return set_error(B2PA_ERR_INVALID_ARGUMENT, "patch_table: null pointer argument");
  if (n_cells > INT32_MAX) return set_error(B2PA_ERR_UNSUPPORTED, "patch_table: more than 2^31 cells");
  return launch_patch_table(table, n_cells, pairs, n_pairs, status, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
