// tma_map.cu -- host-side creation of TMA tensor maps for the block pools.
//
// A pool [num_blocks, H, block_size, D] is viewed as a 2-d tensor of
// num_blocks*H*block_size rows of D elements; one box is one (block, head)
// page restricted to 64 columns (128 bytes), written to shared memory with
// the 128-byte swizzle the UMMA descriptors expect.  The driver entry point
// is resolved through the runtime once, so the library does not link libcuda.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "b2pa.h"
#include "kernels.h"

namespace b2pa {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace

namespace {
// Recently encoded maps: a pool keeps its address until it grows, so the
// maps of the last few pools are reused instead of re-encoded every call.
struct MapKey {
  const void* pool;
  int64_t rows;
  int D, block_size, dtype;
  bool operator==(const MapKey& o) const {
    return pool == o.pool && rows == o.rows && D == o.D && block_size == o.block_size && dtype == o.dtype;
  }
};
constexpr int kMapCache = 16;
std::mutex g_map_mu;
MapKey g_keys[kMapCache];
CUtensorMap g_maps[kMapCache];
int g_next = 0, g_used = 0;
}  // namespace

bool encode_pool_tensor_map_uncached(CUtensorMap* map, const void* pool, int64_t rows, int D, int block_size,
                                     int dtype);

bool encode_pool_tensor_map(CUtensorMap* map, const void* pool, int64_t rows, int D, int block_size, int dtype) {
  const MapKey key{pool, rows, D, block_size, dtype};
  {
    std::lock_guard<std::mutex> g(g_map_mu);
    for (int i = 0; i < g_used; ++i)
      if (g_keys[i] == key) {
        *map = g_maps[i];
        return true;
      }
  }
  if (!encode_pool_tensor_map_uncached(map, pool, rows, D, block_size, dtype)) return false;
  std::lock_guard<std::mutex> g(g_map_mu);
  g_keys[g_next] = key;
  g_maps[g_next] = *map;
  g_next = (g_next + 1) % kMapCache;
  if (g_used < kMapCache) ++g_used;
  return true;
}

// q [B, H, T, D] (element strides sq = {b, h, t}, unit D stride) as a 4-d
// tensor {D, x1, x2, x3}: the outer three are t, h, b ordered by stride, so
// the usual layouts ([B, H, T, D], or the [B, T, H, D] view the model's head
// split makes) are packed maps.  One box is 64 columns (128 bytes) of 128
// consecutive rows t of one (b, h), zero-filled past T, in the 128-byte
// swizzle.  dim_of[0..2]: the map dimension (1..3) holding t, h, b.  False if
// the driver refuses the layout (the kernel then loads q with threads).
bool encode_q_tensor_map(CUtensorMap* map, const void* q, int B, int H, int T, int D, const int64_t sq[3], int dtype,
                         int dim_of[3]) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (dtype != B2PA_DTYPE_BF16 && dtype != B2PA_DTYPE_F16)) return false;
  const int64_t ext[3] = {T, H, B};              // logical t, h, b
  const int64_t str[3] = {sq[2], sq[1], sq[0]};  // their element strides
  int order[3] = {0, 1, 2};                      // logical dims by increasing stride (t first on ties)
  for (int i = 1; i < 3; ++i)
    for (int j = i; j > 0 && str[order[j]] < str[order[j - 1]]; --j) {
      const int x = order[j];
      order[j] = order[j - 1];
      order[j - 1] = x;
    }
  cuuint64_t dims[4] = {(cuuint64_t)D, 0, 0, 0};
  cuuint64_t strides[3];
  cuuint32_t box[4] = {64, 1, 1, 1};
  for (int i = 0; i < 3; ++i) {
    const int l = order[i];
    if (str[l] <= 0) return false;
    dims[i + 1] = (cuuint64_t)ext[l];
    strides[i] = (cuuint64_t)str[l] * 2;
    box[i + 1] = l == 0 ? 128 : 1;
    dim_of[l] = i + 1;
  }
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == B2PA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 4, const_cast<void*>(q), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_pool_tensor_map_uncached(CUtensorMap* map, const void* pool, int64_t rows, int D, int block_size,
                                     int dtype) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || rows <= 0 || rows > ((int64_t)1 << 31)) return false;
  const CUtensorMapDataType dt = dtype == B2PA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)block_size};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace b2pa
