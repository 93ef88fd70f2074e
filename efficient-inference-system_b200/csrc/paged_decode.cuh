// paged_decode.cuh -- single-query paged decode attention for sm_100a.
//
// Replaces the Triton decode kernel of the reference
// (src/kernels/triton_paged_attention.py:10-85, launcher :179-217), which
// runs one program per (sequence, head) and walks every token of the page
// table sequentially.  Semantics follow the torch reference
// (src/kernels/reference_paged_attention.py:31-57): for sequence b the query
// sits at position seq_len - cur_len and sees keys
// 0 .. min(seq_len, seq_len - cur_len + 1) - 1; out = softmax(q.K^T * scale).V
// in fp32, zeros when no key is visible, stored in the element type.
//
// Design (HBM-bound gather, no tensor cores):
//   * work item = (sequence b, head group of G heads, split of P pages).
//     A one-CTA plan kernel turns seq_lens/cur_lens into per-sequence item
//     offsets; a persistent grid (SMs x resident CTAs) strides over items.
//   * per CTA: one producer warp + G consumer warps.  The producer walks the
//     block table and moves, per page, the G contiguous [block_size, D] head
//     pages of K and of V with two cp.async.bulk copies into a ring of
//     shared-memory stages guarded by full/empty mbarriers (no multicast).
//     It also stages the pre-scaled query of the item and a small metadata
//     record, so consumers never touch global memory on the way in.
//   * each consumer warp owns one head: lanes split a page into
//     (row group, 16-byte column chunk); partial q.k dots are reduced with a
//     transpose-reduce (block_size-1 shuffles per page instead of
//     5 x block_size), then an online softmax in the log2 domain updates the
//     fp32 accumulator.
//   * items covering a whole sequence write the output directly; split
//     sequences leave (m, l, acc) partials in the workspace and a combine
//     kernel merges them with a log-sum-exp rescale.
#pragma once

#include <algorithm>
#include <climits>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace b2pa {

// Bytes per lane access: the widest of 16/8/4 for which the rows that one
// warp covers at once (32 / lanes-per-row) fit inside one page.
constexpr int decode_chunk_bytes(int row_bytes, int bs) {
  int cands[3] = {16, 8, 4};
  for (int i = 0; i < 3; ++i) {
    const int cb = cands[i];
    if (row_bytes % cb) continue;
    const int nc = row_bytes / cb;
    const int lpr = nc < 32 ? nc : 32;
    if (nc % lpr) continue;
    if (32 / lpr <= bs) return cb;
  }
  return 0;
}

template <typename T, int D, int BS>
struct DecodeTile {
  static constexpr int ES = (int)sizeof(T);
  static constexpr int ROW_BYTES = D * ES;
  static constexpr int CB = decode_chunk_bytes(ROW_BYTES, BS);
  static_assert(CB > 0, "unsupported (head_dim, block_size)");
  static constexpr int CH = CB / ES;             // elements per lane access
  static constexpr int NC = D / CH;              // accesses per row
  static constexpr int LPR = NC < 32 ? NC : 32;  // lanes per row
  static constexpr int CPL = NC / LPR;           // accesses per lane per row
  static constexpr int RP = 32 / LPR;            // rows covered at once
  static constexpr int NR = BS / RP;             // rows per lane per page
  static_assert(NR >= 1 && NR <= LPR, "row split does not fit the warp");
  static constexpr int SH = ilog2(LPR) - ilog2(NR);
  static constexpr int DUP = LPR / NR;           // lanes holding each score
  static constexpr int HEAD_PAGE_BYTES = BS * ROW_BYTES;
};

struct DecodeParams {
  const void* q;
  int64_t sq_b, sq_h;
  const void* k_pool;
  const void* v_pool;
  int64_t num_blocks;
  const int32_t* page_table;
  int64_t pt_stride;
  int max_pages;
  const int32_t* seq_lens;
  const int32_t* cur_lens;
  void* out;
  int64_t so_b, so_h;
  int B, H, G, HG;
  int pages_per_split;
  // 1: contiguous split -- CTA c streams units [c*W/Gu, (c+1)*W/Gu) of the
  // flattened (sequence, head group, page) sequence; 0: items of
  // pages_per_split pages, strided over the grid.
  int contig;
  int min_units;    // contiguous split: a CTA takes at least this many units
  int grid_launch;  // CTAs launched (the combine kernel recomputes the split from it)
  int stages;
  int stage_bytes;
  int meta_off;  // offset of StageMeta inside a stage
  int q_off;     // offset of the fp32 query block inside a stage
  float qscale;  // scale * log2(e)
  int32_t* item_off;
  int plan_in_smem;  // 1: every CTA computes the item offsets itself (shared memory)
  int off_smem;      // byte offset of those offsets in dynamic shared memory
  float* part_ml;
  float* part_acc;
  int32_t* status;
  // Fused KV append (null app_len: none); see decode_append_rows.
  const void* k_new;
  const void* v_new;
  int64_t skn_b, skn_h, svn_b, svn_h;
  const int32_t* app_start;
  const int32_t* app_len;
  int app_vb;
  int64_t* seq_out;
};

struct StageMeta {
  int b;
  int h0;
  int item;
  int nsplit;
  int nvalid;  // visible tokens of this page (0 = skip)
  int flags;
  int pad[2];
};
constexpr int kFirst = 1;
constexpr int kLast = 2;
constexpr int kEnd = 4;  // the CTA's last item

// Visible key count of sequence b, clamped to the page table width.
__device__ __forceinline__ int decode_visible(const DecodeParams& p, int b, int bs) {
  const int64_t L = p.seq_lens[b];
  const int64_t c = p.cur_lens[b];
  int64_t e = L - c + 1;
  e = e < L ? e : L;
  if (e < 0) e = 0;
  const int64_t cap = (int64_t)p.max_pages * bs;
  if (e > cap) e = cap;
  return (int)e;
}

// Offsets counted per sequence b: HG * number of items (splits of
// pages_per_split pages, at least one), or for the contiguous split HG *
// units (visible pages, at least one, so that a stream with no visible key
// still writes its zeros).
template <int BS>
__device__ __forceinline__ int decode_items_of(const DecodeParams& p, int b) {
  const int vis = decode_visible(p, b, BS);
  const int np = (vis + BS - 1) / BS;
  const int n = p.contig ? np : (np + p.pages_per_split - 1) / p.pages_per_split;
  return (n < 1 ? 1 : n) * p.HG;
}

// The contiguous split (32-bit arithmetic: the host keeps B * HG *
// max_pages below 2^31).  Gu = CTAs in use, about one per min_units units,
// at least one, at most the launch.  With q = W / Gu and r = W % Gu, CTA c
// takes q units, plus one for the first r CTAs; its first unit is
// c*q + min(c, r) (Gu <= W, so q >= 1).  decode_cta_of inverts it;
// decode_slot is the partial slot of the piece of a stream starting at unit
// `sstart` that CTA c holds: 2c when the stream reaches back to the CTA's
// first unit (its first piece), else 2c + 1 (only these two can be cut).
__device__ __forceinline__ int decode_ctas_used(const DecodeParams& p, int W) {
  int g = W / p.min_units + (W % p.min_units != 0);
  if (g > p.grid_launch) g = p.grid_launch;
  return g < 1 ? 1 : g;
}
__device__ __forceinline__ int decode_start(int c, int W, int Gu) {
  const int q = W / Gu, r = W - (W / Gu) * Gu;
  return c * q + (c < r ? c : r);
}
__device__ __forceinline__ int decode_cta_of(int w, int W, int Gu) {
  const int q = W / Gu, r = W - (W / Gu) * Gu;
  const int big = r * (q + 1);
  return w < big ? w / (q + 1) : r + (w - big) / q;
}
__device__ __forceinline__ int decode_slot(int c, int sstart, int W, int Gu) {
  return 2 * c + (sstart > decode_start(c, W, Gu) ? 1 : 0);
}

// One CTA: item_off[b] = prefix of decode_items_of, item_off[B] = total.
template <int BS>
__global__ void __launch_bounds__(1024) decode_plan_kernel(DecodeParams p) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < p.B; base += 1024) {
    const int b = base + tid;
    int n = 0;
    if (b < p.B) {
      const int64_t L = p.seq_lens[b];
      if (L > (int64_t)p.max_pages * BS) set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
      n = decode_items_of<BS>(p, b);
    }
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFullMask, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFullMask, w, o);
        if (lane >= o) w += y;
      }
      warp_sums[lane] = w;  // inclusive
    }
    __syncthreads();
    const int excl = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + x - n;
    if (b < p.B) p.item_off[b] = excl;
    __syncthreads();
    if (tid == 0) carry += warp_sums[31];
    __syncthreads();
  }
  if (tid == 0) p.item_off[p.B] = carry;
}

// The plan of decode_plan_kernel computed by one CTA of the decode kernel
// (all its threads): off[b] = exclusive prefix of the item counts, off[B] =
// total.  CTA 0 also publishes it to p.item_off for the combine kernel and
// reports lengths past the page table.
template <int BS>
__device__ void decode_plan_cta(const DecodeParams& p, int* off) {
  __shared__ int warp_tot[32];
  const int nt = blockDim.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  int carry = 0;
  for (int base = 0; base < p.B; base += nt) {
    const int b = base + tid;
    int n = 0;
    if (b < p.B) {
      n = decode_items_of<BS>(p, b);
      if (blockIdx.x == 0 && (int64_t)p.seq_lens[b] > (int64_t)p.max_pages * BS) set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
    }
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFullMask, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    int before = 0, all = 0;
    for (int w2 = 0; w2 < nw; ++w2) {
      const int t = warp_tot[w2];
      before += w2 < warp ? t : 0;
      all += t;
    }
    if (b < p.B) {
      off[b] = carry + before + x - n;
      if (blockIdx.x == 0) p.item_off[b] = carry + before + x - n;
    }
    carry += all;
    __syncthreads();
  }
  if (tid == 0) {
    off[p.B] = carry;
    if (blockIdx.x == 0) p.item_off[p.B] = carry;
  }
  __syncthreads();
}

// Reduces v[0..N) over the M lanes (xor masks M/2..1) of a lane group so
// that lane c ends up with the full sum of element (c >> (log2 M - log2 N)).
template <int N, int M>
struct TransposeReduce {
  __device__ __forceinline__ static float run(float (&v)[N], int c) {
    if constexpr (M == 1) {
      return v[0];
    } else if constexpr (N == 1) {
      float x = v[0];
#pragma unroll
      for (int m = M / 2; m >= 1; m >>= 1) x += __shfl_xor_sync(kFullMask, x, m);
      return x;
    } else {
      constexpr int H = N / 2;
      constexpr int MASK = M / 2;
      const bool upper = (c & MASK) != 0;
      float w[H];
#pragma unroll
      for (int k = 0; k < H; ++k) {
        const float send = upper ? v[k] : v[k + H];
        const float keep = upper ? v[k + H] : v[k];
        w[k] = keep + __shfl_xor_sync(kFullMask, send, MASK);
      }
      return TransposeReduce<H, M / 2>::run(w, c);
    }
  }
};

// Copies the new K and V rows of heads h0 .. h0+G-1 of sequence b to pool
// row `off` of block `blk`, VB bytes per access, spread over the warp.
template <int VB, int ROW_BYTES, int BS>
__device__ __forceinline__ void decode_copy_new_rows(const DecodeParams& p, int b, int h0, int G, int64_t blk,
                                                     int off, int lane, int es) {
  using W = typename VecWord<VB>::type;
  constexpr int CPR = ROW_BYTES / VB;  // accesses per head row
  const char* ks = static_cast<const char*>(p.k_new);
  const char* vs = static_cast<const char*>(p.v_new);
  char* kp = const_cast<char*>(static_cast<const char*>(p.k_pool));
  char* vp = const_cast<char*>(static_cast<const char*>(p.v_pool));
  for (int i = lane; i < G * CPR; i += 32) {
    const int hh = i / CPR;
    const int c = i - hh * CPR;
    const int h = h0 + hh;
    const int64_t src_k = ((int64_t)b * p.skn_b + (int64_t)h * p.skn_h) * es + (int64_t)c * VB;
    const int64_t src_v = ((int64_t)b * p.svn_b + (int64_t)h * p.svn_h) * es + (int64_t)c * VB;
    const int64_t dst = ((blk * p.H + h) * BS + off) * (int64_t)ROW_BYTES + (int64_t)c * VB;
    const W kw = *reinterpret_cast<const W*>(ks + src_k);
    const W vw = *reinterpret_cast<const W*>(vs + src_v);
    *reinterpret_cast<W*>(kp + dst) = kw;
    *reinterpret_cast<W*>(vp + dst) = vw;
  }
}

// The KV append fused into the decode launch (b2pa_paged_decode_append),
// run by the producer warp at the start of the LAST split of (sequence b,
// head group h0/G), before it issues any copy of that split's pages: the new
// token sits at app_start[b] = seq_len - 1, so when it is visible it lies in
// the last visible page, which belongs to this split; when it is not visible
// (cur_len >= 2) nothing in the launch reads it.  No other item copies the
// (block, head) pages of these heads.  Each lane's proxy fence orders its
// generic-proxy stores before the bulk (async-proxy) copies that lane 0
// issues after the warp barrier.  A row whose position is not seq_len - 1
// (it could sit in another split's page) is skipped and reported as an
// invalid argument; position and block checks otherwise follow
// kv_append_kernel: out-of-range writes are skipped and reported.
template <typename T, int D, int BS>
__device__ __forceinline__ void decode_append_rows(const DecodeParams& p, int b, int h0, int G, int lane) {
  if (p.app_len[b] > 0) {
    const int64_t pos = p.app_start[b];
    const int64_t page = pos / BS;
    int64_t blk = -1;
    if (pos >= 0 && page < p.max_pages) blk = p.page_table[(int64_t)b * p.pt_stride + page];
    if (pos != (int64_t)p.seq_lens[b] - 1) {
      if (lane == 0) set_status(p.status, B2PA_ERR_INVALID_ARGUMENT);
    } else if (blk < 0 || blk >= p.num_blocks) {
      if (lane == 0) set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
    } else {
      constexpr int ES = (int)sizeof(T);
      constexpr int RB = D * ES;
      const int off = (int)(pos - page * BS);
      if (p.app_vb == 16) {
        if constexpr (RB % 16 == 0) decode_copy_new_rows<16, RB, BS>(p, b, h0, G, blk, off, lane, ES);
      } else if (p.app_vb == 8) {
        if constexpr (RB % 8 == 0) decode_copy_new_rows<8, RB, BS>(p, b, h0, G, blk, off, lane, ES);
      } else {
        decode_copy_new_rows<4, RB, BS>(p, b, h0, G, blk, off, lane, ES);
      }
      fence_proxy_async_global();
    }
  }
  __syncwarp();
}

template <typename T, int D, int BS>
__global__ void __launch_bounds__(160) paged_decode_kernel(DecodeParams p) {
  using Tile = DecodeTile<T, D, BS>;
  using V = Vec<T, Tile::CH>;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)p.stages * p.stage_bytes);
  uint64_t* empty = full + p.stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], G);
    }
    fence_mbar_init();
  }
  // Launched programmatically after the KV append: nothing below may read
  // the pools (or anything else an earlier kernel writes) before this.
  pdl_wait();
  const int* off = p.item_off;
  if (p.plan_in_smem) {
    int* s_off = reinterpret_cast<int*>(smem + p.off_smem);
    decode_plan_cta<BS>(p, s_off);  // ends with __syncthreads
    off = s_off;
  } else {
    __syncthreads();
  }

  const int total = off[p.B];
  const int chunk_bytes = G * Tile::HEAD_PAGE_BYTES;

  if (warp == G) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0, issued_par = 0;  // per-stage bookkeeping for drain
    int cur_b = 0;
    bool ok = true;
    // Item split: item w, then w + gridDim.x, ...  Contiguous split: the
    // units [u, uend) of this CTA, one piece (a run of units of one stream)
    // at a time.
    int w = blockIdx.x, u = 0, uend = 0, Gu = 1;
    if (p.contig) {
      Gu = decode_ctas_used(p, total);
      if ((int)blockIdx.x < Gu) {
        u = decode_start(blockIdx.x, total, Gu);
        uend = decode_start(blockIdx.x + 1, total, Gu);
      }
    }
    while (ok && (p.contig ? u < uend : w < total)) {
      const int key = p.contig ? u : w;
      // Locate the sequence of unit/item `key` (visited in increasing order).
      while (true) {
        const int idx = cur_b + 1 + lane;
        const int v = idx <= p.B ? off[idx] : INT_MAX;
        const unsigned m = __ballot_sync(kFullMask, v > key);
        if (m) {
          cur_b += __ffs(m) - 1;
          break;
        }
        cur_b += 32;
      }
      const int b = cur_b;
      const int off0 = off[b];
      const int per = (off[b + 1] - off0) / p.HG;  // items or units per stream
      const int r = key - off0;
      const int hg = r / per;
      const int s = r - hg * per;
      const int vis = decode_visible(p, b, BS);
      const int npages = (vis + BS - 1) / BS;
      int p0, span, count, item, nsplit, flags_end = 0;
      bool stream_tail;  // the piece holds the stream's last page
      if (p.contig) {
        // Units s .. se-1 of the stream are pages s .. se-1 (one unit and
        // no page when nothing is visible).
        const int left = uend - u;
        const int se = per - s < left ? per : s + left;
        p0 = s;
        span = se - s;
        count = span;
        const bool whole = s == 0 && se == per;
        item = whole ? 0 : decode_slot(blockIdx.x, u - s, total, Gu);
        nsplit = whole ? 1 : 2;
        stream_tail = se == per;
        if (u + count == uend) flags_end = kEnd;
        u += count;
      } else {
        p0 = s * p.pages_per_split;
        span = p.pages_per_split;
        item = w;
        nsplit = per;
        stream_tail = s == per - 1;
        w += gridDim.x;
      }
      int p1 = p0 + span;
      p1 = p1 < npages ? p1 : npages;
      const int npg = p1 > p0 ? p1 - p0 : 0;
      if (!p.contig) count = npg > 0 ? npg : 1;
      const int h0 = hg * G;
      const char* kbase = static_cast<const char*>(p.k_pool);
      const char* vbase = static_cast<const char*>(p.v_pool);
      if (p.app_len != nullptr && stream_tail) decode_append_rows<T, D, BS>(p, b, h0, G, lane);

      for (int i0 = 0; i0 < count && ok; i0 += 32) {
        int blk = -1;
        if (i0 + lane < npg) {
          blk = p.page_table[(int64_t)b * p.pt_stride + p0 + i0 + lane];
          if (blk >= p.num_blocks) {
            set_status(p.status, B2PA_ERR_BAD_BLOCK_ID);
            blk = -1;
          }
        }
        const int nj = count - i0 < 32 ? count - i0 : 32;
        for (int j = 0; j < nj; ++j) {
          const int bj = __shfl_sync(kFullMask, blk, j);
          // Every lane waits (and so acquires the consumers' release); the
          // vote keeps the warp converged if the bounded wait gives up.
          if (!__all_sync(kFullMask, mbar_wait_bounded(&empty[stage], phase ^ 1, p.status))) {
            ok = false;
            break;
          }
          unsigned char* st = smem + (size_t)stage * p.stage_bytes;
          const int pi = i0 + j;
          // The page copies go out first; the query and the metadata record
          // are written while they are in flight, and the arrival that lets
          // the consumers in comes after both (the barrier completes once the
          // arrival and all expected bytes are in).
          if (lane == 0 && bj >= 0) {
            mbar_expect_tx(&full[stage], 2u * chunk_bytes);
            const int64_t src = ((int64_t)bj * p.H + h0) * Tile::HEAD_PAGE_BYTES;
            bulk_g2s(st, kbase + src, chunk_bytes, &full[stage]);
            bulk_g2s(st + chunk_bytes, vbase + src, chunk_bytes, &full[stage]);
          }
          if (pi == 0) {
            // Stage the query of this item, pre-scaled, as fp32.
            float* qs = reinterpret_cast<float*>(st + p.q_off);
            const T* qg = static_cast<const T*>(p.q);
            for (int e = lane; e < G * D; e += 32) {
              const int hh = e / D;
              const int d = e - hh * D;
              qs[e] = to_f32(qg[(int64_t)b * p.sq_b + (int64_t)(h0 + hh) * p.sq_h + d]) * p.qscale;
            }
          }
          if (lane == 0) {
            StageMeta* meta = reinterpret_cast<StageMeta*>(st + p.meta_off);
            int nv = 0;
            if (bj >= 0) {
              nv = vis - (p0 + pi) * BS;
              nv = nv < BS ? nv : BS;
              nv = nv > 0 ? nv : 0;
            }
            meta->b = b;
            meta->h0 = h0;
            meta->item = item;
            meta->nsplit = nsplit;
            meta->nvalid = nv;
            meta->flags = (pi == 0 ? kFirst : 0) | (pi == count - 1 ? kLast | flags_end : 0);
          }
          __threadfence_block();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[stage]);
          issued |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    if (p.seq_out != nullptr && blockIdx.x == 0)
      for (int b = lane; b < p.B; b += 32) p.seq_out[b] = p.seq_lens[b];
    pdl_launch_dependents();
    if (!ok && lane == 0) {
      // Gave up: let every copy this CTA started land before exiting.
      for (int s2 = 0; s2 < p.stages; ++s2)
        if (issued & (1u << s2)) mbar_wait_bounded(&full[s2], (issued_par >> s2) & 1u, p.status);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int rg = lane / Tile::LPR;
  const int c = lane - rg * Tile::LPR;
  const int r_own = rg + Tile::RP * (c >> Tile::SH);
  int stage = 0;
  uint32_t phase = 0;
  // Item split: the producer's items w = blockIdx.x, + gridDim.x, ...
  // Contiguous split: pieces until the one flagged kEnd (none for a CTA past
  // the ones in use).
  int w = blockIdx.x;
  bool more = p.contig ? (int)blockIdx.x < decode_ctas_used(p, total) : w < total;
  while (more) {
    float q[Tile::CPL][Tile::CH];
    float acc[Tile::CPL][Tile::CH];
    float m = -INFINITY, l_part = 0.f;
    while (true) {
      if (!__all_sync(kFullMask, mbar_wait_bounded(&full[stage], phase, p.status))) return;
      const unsigned char* st = smem + (size_t)stage * p.stage_bytes;
      const StageMeta meta = *reinterpret_cast<const StageMeta*>(st + p.meta_off);
      if (meta.flags & kFirst) {
        const float* qs = reinterpret_cast<const float*>(st + p.q_off) + warp * D;
#pragma unroll
        for (int j = 0; j < Tile::CPL; ++j)
#pragma unroll
          for (int e = 0; e < Tile::CH; ++e) {
            q[j][e] = qs[(c + Tile::LPR * j) * Tile::CH + e];
            acc[j][e] = 0.f;
          }
        m = -INFINITY;
        l_part = 0.f;
      }
      const int nvalid = meta.nvalid;
      if (nvalid > 0) {
        const unsigned char* kb = st + warp * Tile::HEAD_PAGE_BYTES;
        const unsigned char* vb = kb + chunk_bytes;
        float s[Tile::NR];
#pragma unroll
        for (int i = 0; i < Tile::NR; ++i) {
          const int row = rg + Tile::RP * i;
          float a = 0.f;
#pragma unroll
          for (int j = 0; j < Tile::CPL; ++j) {
            V kv;
            kv.w = ld_shared<typename V::Word>(kb + row * Tile::ROW_BYTES + (c + Tile::LPR * j) * Tile::CB);
            float kf[Tile::CH];
            kv.to_float(kf);
#pragma unroll
            for (int e = 0; e < Tile::CH; ++e) a = fmaf(q[j][e], kf[e], a);
          }
          s[i] = a;
        }
        float sc = TransposeReduce<Tile::NR, Tile::LPR>::run(s, c);
        if (r_own >= nvalid) sc = -INFINITY;
        const float m_new = fmaxf(m, warp_max(sc));
        const float alpha = exp2f(m - m_new);
        const float p_own = exp2f(sc - m_new);
        l_part = l_part * alpha + p_own;
#pragma unroll
        for (int j = 0; j < Tile::CPL; ++j)
#pragma unroll
          for (int e = 0; e < Tile::CH; ++e) acc[j][e] *= alpha;
#pragma unroll
        for (int i = 0; i < Tile::NR; ++i) {
          const float pi = __shfl_sync(kFullMask, p_own, rg * Tile::LPR + (i << Tile::SH));
          const int row = rg + Tile::RP * i;
          if (row < nvalid) {
#pragma unroll
            for (int j = 0; j < Tile::CPL; ++j) {
              V vv;
              vv.w = ld_shared<typename V::Word>(vb + row * Tile::ROW_BYTES + (c + Tile::LPR * j) * Tile::CB);
              float vf[Tile::CH];
              vv.to_float(vf);
#pragma unroll
              for (int e = 0; e < Tile::CH; ++e) acc[j][e] = fmaf(pi, vf[e], acc[j][e]);
            }
          }
        }
        m = m_new;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == p.stages) {
        stage = 0;
        phase ^= 1;
      }
      if (meta.flags & kLast) {
        // Merge the row groups, then the per-lane denominators.
#pragma unroll
        for (int mk = Tile::LPR; mk < 32; mk <<= 1)
#pragma unroll
          for (int j = 0; j < Tile::CPL; ++j)
#pragma unroll
            for (int e = 0; e < Tile::CH; ++e) acc[j][e] += __shfl_xor_sync(kFullMask, acc[j][e], mk);
        const float l = warp_sum(l_part) * (1.0f / Tile::DUP);
        const int h = meta.h0 + warp;
        if (meta.nsplit == 1) {
          const float den = fmaxf(l, 1e-9f);
          if (rg == 0) {
            T* o = static_cast<T*>(p.out) + (int64_t)meta.b * p.so_b + (int64_t)h * p.so_h;
#pragma unroll
            for (int j = 0; j < Tile::CPL; ++j) {
              float f[Tile::CH];
#pragma unroll
              for (int e = 0; e < Tile::CH; ++e) f[e] = acc[j][e] / den;
              V ov;
              ov.from_float(f);
              *reinterpret_cast<typename V::Word*>(o + (c + Tile::LPR * j) * Tile::CH) = ov.w;
            }
          }
        } else {
          const int64_t slot = (int64_t)meta.item * G + warp;
          if (rg == 0) {
            float* pa = p.part_acc + slot * D;
#pragma unroll
            for (int j = 0; j < Tile::CPL; ++j)
#pragma unroll
              for (int e = 0; e < Tile::CH; ++e) pa[(c + Tile::LPR * j) * Tile::CH + e] = acc[j][e];
          }
          if (lane == 0) {
            p.part_ml[2 * slot] = m;
            p.part_ml[2 * slot + 1] = l;
          }
        }
        if (p.contig) {
          more = (meta.flags & kEnd) == 0;
        } else {
          w += gridDim.x;
          more = w < total;
        }
        break;
      }
    }
  }
}

// One warp per (sequence, head) whose stream was split: log-sum-exp merge.
// The split statistics are read one split per lane and reduced across the
// warp, and the partial accumulators are read with independent loads (the
// weights come by shuffle), so the merge is not a chain of dependent loads.
// Item split: the stream's splits are items base .. base+nsplit-1.
// Contiguous split: its pieces are held by CTAs c0 .. c1 (the CTAs of its
// first and last unit), piece j in slot decode_slot(c0 + j, ...); a stream
// inside one CTA was written directly.
template <typename T, int D>
__global__ void __launch_bounds__(256) decode_combine_kernel(DecodeParams p) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (gw >= (int64_t)p.B * p.H) return;
  const int b = (int)(gw / p.H);
  const int h = (int)(gw - (int64_t)b * p.H);
  const int off0 = p.item_off[b];
  const int per = (p.item_off[b + 1] - off0) / p.HG;
  const int hg = h / p.G;
  const int hi = h - hg * p.G;
  const int64_t base = (int64_t)off0 + (int64_t)hg * per;  // the stream's first item / unit
  int nsplit = per, c0 = 0, W = 0, Gu = 1;
  if (p.contig) {
    W = p.item_off[p.B];
    Gu = decode_ctas_used(p, W);
    c0 = decode_cta_of((int)base, W, Gu);
    nsplit = decode_cta_of((int)base + per - 1, W, Gu) - c0 + 1;
  }
  if (nsplit <= 1) return;
  auto slot_of = [&](int s) -> int64_t {
    return p.contig ? (int64_t)decode_slot(c0 + s, (int)base, W, Gu) : base + s;
  };
  float M = -INFINITY;
  for (int s = lane; s < nsplit; s += 32) M = fmaxf(M, p.part_ml[2 * (slot_of(s) * p.G + hi)]);
  M = warp_max(M);
  constexpr int PER = D >= 32 ? D / 32 : 1;
  float o[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) o[i] = 0.f;
  float L = 0.f;
  for (int s0 = 0; s0 < nsplit; s0 += 32) {
    const int s = s0 + lane;
    float wl = 0.f;
    if (s < nsplit) {
      const int64_t slot = slot_of(s) * p.G + hi;
      const float ms = p.part_ml[2 * slot];
      wl = (M == -INFINITY) ? 0.f : exp2f(ms - M);
      L = fmaf(p.part_ml[2 * slot + 1], wl, L);
    }
    const int cnt = nsplit - s0 < 32 ? nsplit - s0 : 32;
#pragma unroll 4
    for (int j = 0; j < cnt; ++j) {
      const float wgt = __shfl_sync(kFullMask, wl, j);
      const float* pa = p.part_acc + (slot_of(s0 + j) * p.G + hi) * D;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int d = lane + 32 * i;
        if (d < D) o[i] = fmaf(wgt, pa[d], o[i]);
      }
    }
  }
  L = warp_sum(L);
  const float den = fmaxf(L, 1e-9f);
  T* out = static_cast<T*>(p.out) + (int64_t)b * p.so_b + (int64_t)h * p.so_h;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int d = lane + 32 * i;
    if (d < D) out[d] = from_f32<T>(o[i] / den);
  }
}

int decode_occupancy_cached(const void* func, int threads, size_t smem);

template <typename T, int D, int BS>
int launch_decode_impl(const AttnArgs& a, const DecodePlan& plan, cudaStream_t stream) {
  using Tile = DecodeTile<T, D, BS>;
  DecodeParams p;
  p.q = a.q;
  p.sq_b = a.sq[0];
  p.sq_h = a.sq[1];
  p.k_pool = a.k_pool;
  p.v_pool = a.v_pool;
  p.num_blocks = a.num_blocks;
  p.page_table = a.page_table;
  p.pt_stride = a.pt_stride;
  p.max_pages = a.max_pages;
  p.seq_lens = a.seq_lens;
  p.cur_lens = a.cur_lens;
  p.out = a.out;
  p.so_b = a.so[0];
  p.so_h = a.so[1];
  p.B = a.B;
  p.H = a.H;
  p.G = plan.G;
  p.HG = plan.HG;
  p.pages_per_split = plan.pages_per_split;
  p.contig = plan.contig;
  p.min_units = kDecodeMinUnits;
  p.qscale = a.scale * kLog2e;
  char* ws = static_cast<char*>(a.workspace);
  p.item_off = reinterpret_cast<int32_t*>(ws + plan.off_item_off);
  p.part_ml = reinterpret_cast<float*>(ws + plan.off_part_ml);
  p.part_acc = reinterpret_cast<float*>(ws + plan.off_part_acc);
  p.status = a.status;
  p.k_new = a.k_new;
  p.v_new = a.v_new;
  p.skn_b = a.skn[0];
  p.skn_h = a.skn[1];
  p.svn_b = a.svn[0];
  p.svn_h = a.svn[1];
  p.app_start = a.app_start;
  p.app_len = a.app_len;
  p.app_vb = a.app_vb;
  p.seq_out = a.seq_out;

  const int chunk = plan.G * Tile::HEAD_PAGE_BYTES;
  p.q_off = 2 * chunk;
  p.meta_off = p.q_off + plan.G * D * 4;
  p.stage_bytes = (p.meta_off + (int)sizeof(StageMeta) + 127) / 128 * 128;
  int stages = (96 * 1024) / p.stage_bytes;
  stages = std::max(2, std::min(8, stages));
  const int max_smem = device_max_smem_optin();
  while (stages > 2 && (size_t)stages * p.stage_bytes + 16 * stages > (size_t)max_smem) --stages;
  p.stages = stages;
  // Item offsets in shared memory (every CTA computes them) when they fit;
  // otherwise the one-CTA plan kernel writes them to the workspace.
  p.off_smem = stages * p.stage_bytes + 16 * stages;
  const size_t off_bytes = ((size_t)(a.B + 1) * 4 + 15) / 16 * 16;
  p.plan_in_smem = off_bytes <= 32 * 1024 && (size_t)p.off_smem + off_bytes <= (size_t)max_smem ? 1 : 0;
  const size_t smem = (size_t)p.off_smem + (p.plan_in_smem ? off_bytes : 0);
  if (smem > (size_t)max_smem)
    return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode: %zu bytes of shared memory exceed the device limit", smem);
  const int threads = (plan.G + 1) * 32;

  auto kern = paged_decode_kernel<T, D, BS>;
  int rc_attr = set_max_dynamic_smem_cached(reinterpret_cast<const void*>(kern), (int)smem);
  if (rc_attr != B2PA_OK) return rc_attr;
  cudaError_t e;
  const int per_sm = decode_occupancy_cached(reinterpret_cast<const void*>(kern), threads, smem);
  if (per_sm <= 0) return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode: kernel does not fit on an SM");
  int64_t grid = (int64_t)device_sm_count() * per_sm;
  // Contiguous split: two partial slots per CTA; item split: no more CTAs
  // than items.
  const int64_t cap = plan.contig ? plan.max_items / 2 : plan.max_items;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  p.grid_launch = (int)grid;

  if (!p.plan_in_smem) decode_plan_kernel<BS><<<1, 1024, 0, stream>>>(p);
  e = launch_pdl(kern, dim3((unsigned)grid), dim3(threads), smem, stream, p);
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_decode launch: %s", cudaGetErrorString(e));
  if (plan.contig || plan.max_items > (int64_t)a.B * plan.HG) {  // some stream may be split
    const int64_t warps = (int64_t)a.B * a.H;
    const unsigned cgrid = (unsigned)((warps + 7) / 8);
    e = launch_pdl(decode_combine_kernel<T, D>, dim3(cgrid), dim3(256), 0, stream, p);
    if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_decode combine launch: %s", cudaGetErrorString(e));
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(B2PA_ERR_CUDA, "paged_decode launch: %s", cudaGetErrorString(e));
  return B2PA_OK;
}

template <typename T>
int dispatch_decode(const AttnArgs& a, const DecodePlan& plan, cudaStream_t s) {
#define B2PA_DEC_CASE(DD, BB) \
  if (a.D == DD && a.block_size == BB) return launch_decode_impl<T, DD, BB>(a, plan, s);
#define B2PA_DEC_D(DD) B2PA_DEC_CASE(DD, 8) B2PA_DEC_CASE(DD, 16) B2PA_DEC_CASE(DD, 32)
  B2PA_DEC_D(16)
  B2PA_DEC_D(32)
  B2PA_DEC_D(64)
  B2PA_DEC_D(128)
  B2PA_DEC_D(256)
#undef B2PA_DEC_D
#undef B2PA_DEC_CASE
  return set_error(B2PA_ERR_UNSUPPORTED, "paged_decode: head_dim %d / block_size %d not built", a.D, a.block_size);
}

}  // namespace b2pa
