/*
 * paged_oracle.c -- TEST INFRASTRUCTURE, not part of the product.
 *
 * CPU restatement of the reference's torch paged attention
 * (jacobzhang22/efficient-inference-system,
 *  src/kernels/reference_paged_attention.py:10-59), used only by tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg as the checker and
 * the timed CPU baseline.  Nothing in the b2pa package links or calls it.
 *
 * Algorithm, per (sequence b, head h, query row t), exactly as the reference
 * loops (reference_paged_attention.py:31-57):
 *   past = seq_len[b] - cur_len[b]                       (:32-33)
 *   pos  = past + t                                      (:36)
 *   for token j = 0 .. seq_len-1, stopping at j > pos:   (:40-42)
 *       block = block_ids[j / block_size], off = j % block_size   (:44-45)
 *       score_j = dot(q[b,h,t,:], K[block,h,off,:]) * scale        (:46-48)
 *   no token -> output row stays 0                       (:16, :51-52)
 *   w = softmax(score) (max-subtracted, as torch.softmax) (:54-55)
 *   out[b,h,t,:] = sum_j w_j * V[block,h,off,:]          (:56-57)
 * in float32, like the reference's float32 tensors.  Rows are independent;
 * they are spread over `nthreads` POSIX threads (0 = all online CPUs).
 *
 * Build: oracle/Makefile (gcc -O2 -shared -pthread).
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

typedef struct {
  const float* q;
  const int64_t* qs;
  const float* k_pool;
  const float* v_pool;
  int64_t num_blocks;
  int H, BS, D, B, T;
  const int32_t* block_ids;
  const int64_t* bt_off;
  const int32_t* seq_lens;
  const int32_t* cur_lens;
  float* out;
  float scale;
  atomic_llong next;  /* next row to take */
  atomic_int bad;
} Job;

/* One (b, h, t) row of reference_paged_attention.py:35-57. */
static void attend_row(Job* j, int64_t r, float* sc) {
  const int H = j->H, T = j->T, D = j->D, BS = j->BS;
  const int b = (int)(r / ((int64_t)H * T));
  const int h = (int)((r / T) % H);
  const int t = (int)(r % T);
  float* o = j->out + r * D;
  memset(o, 0, sizeof(float) * (size_t)D);
  const int64_t seq_len = j->seq_lens[b];
  const int64_t pos = seq_len - (int64_t)j->cur_lens[b] + t;
  const int64_t n = seq_len < pos + 1 ? seq_len : pos + 1;
  if (n <= 0) return;
  const float* qv = j->q + b * j->qs[0] + h * j->qs[1] + t * j->qs[2];
  float mx = -INFINITY;
  for (int64_t k = 0; k < n; ++k) {
    const int32_t blk = j->block_ids[j->bt_off[b] + k / BS];
    if (blk < 0 || blk >= j->num_blocks) {
      atomic_store(&j->bad, 1);
      sc[k] = -INFINITY;
      continue;
    }
    const float* kv = j->k_pool + (((int64_t)blk * H + h) * BS + k % BS) * D;
    float dot = 0.f;
    for (int d = 0; d < D; ++d) dot += qv[d * j->qs[3]] * kv[d];
    sc[k] = dot * j->scale;
    if (sc[k] > mx) mx = sc[k];
  }
  float sum = 0.f;
  for (int64_t k = 0; k < n; ++k) {
    sc[k] = expf(sc[k] - mx);
    sum += sc[k];
  }
  for (int64_t k = 0; k < n; ++k) {
    const int32_t blk = j->block_ids[j->bt_off[b] + k / BS];
    if (blk < 0 || blk >= j->num_blocks) continue;
    const float w = sc[k] / sum;
    const float* vv = j->v_pool + (((int64_t)blk * H + h) * BS + k % BS) * D;
    for (int d = 0; d < D; ++d) o[d] += w * vv[d];
  }
}

static void* worker(void* arg) {
  Job* j = (Job*)arg;
  const int64_t rows = (int64_t)j->B * j->H * j->T;
  int64_t cap = 0;
  for (int b = 0; b < j->B; ++b)
    if (j->seq_lens[b] > cap) cap = j->seq_lens[b];
  float* sc = (float*)malloc(sizeof(float) * (size_t)(cap > 0 ? cap : 1));
  for (;;) {
    const int64_t r = atomic_fetch_add(&j->next, 1);
    if (r >= rows) break;
    attend_row(j, r, sc);
  }
  free(sc);
  return NULL;
}

/* q: [B,H,T,D] with element strides qs[4]; pools contiguous [NB,H,BS,D];
 * block_ids: concatenation of every sequence's block list, row b starting at
 * bt_off[b]; out: contiguous [B,H,T,D], written in full.  Returns 0, or -3 if
 * a block id lies outside the pool. */
int oracle_paged_attention_f32(const float* q, const int64_t* qs, const float* k_pool, const float* v_pool,
                               int64_t num_blocks, int H, int BS, int D, const int32_t* block_ids,
                               const int64_t* bt_off, const int32_t* seq_lens, const int32_t* cur_lens,
                               float* out, int B, int T, float scale, int nthreads) {
  Job j = {q, qs, k_pool, v_pool, num_blocks, H, BS, D, B, T, block_ids, bt_off, seq_lens, cur_lens, out, scale};
  atomic_init(&j.next, 0);
  atomic_init(&j.bad, 0);
  if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  int started = 0;
  for (int i = 1; i < nthreads; ++i)
    if (pthread_create(&th[started], NULL, worker, &j) == 0) ++started;
  worker(&j);
  for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
  return atomic_load(&j.bad) ? -3 : 0;
}

/* Threads the oracle uses when asked for 0: the online CPUs. */
int oracle_max_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}
