/*
 * pa_oracle.c -- CPU oracle for the paged-attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: it is compiled into
 * oracle/_build/libpa_oracle.so and loaded by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline / --impl reference
 * legs.  The product (libpa_b200.so and the torch shim) never links it and
 * never falls back to it.
 *
 * Every function restates a reference algorithm in plain scalar C, in the
 * reference's own loop order and float (fp32) arithmetic, and cites the
 * reference file:line it follows (paths relative to the gb10-attn project):
 *
 *   pao_decode            rocm/hip/paged_attn_v1_hip.cpp:104-141  (cpu_reference,
 *                         the reference's only full CPU paged decode)
 *   pao_decode_split      kernels/paged_attn_v3.cu:33-123 (split pass) and
 *                         :128-166 (log-sum-exp merge), scalar restatement
 *   pao_prefill           kernels/paged_attn_prefill.cu:55-74 (causal bound,
 *                         padded rows -> 0) applied to the cpu_reference math
 *   pao_choose_num_splits kernels/paged_attn_v3.cu:170-190 (integer, bit-exact)
 *   pao_dot / pao_scores / pao_softmax
 *                         arm_cpu/src/scalar.cpp:9-46 (scalar dot, scores loop,
 *                         softmax) -- pinned bit-for-bit against that file
 *                         compiled from the reference sources
 *
 * Empty rows: cpu_reference with ctx == 0 divides 0 by 0 and yields NaN; the
 * v3 GPU kernel yields NaN for ctx <= 0 too (m = -3e38, l = 0 in every split,
 * paged_attn_v3.cu:70-77,160-165).  The oracle returns NaN for ctx <= 0 (the
 * reference's std::vector<float>(n) would throw for n < 0).
 *
 * Build: gcc -O3 -fno-tree-vectorize -fPIC -shared (scalar, like
 * arm_cpu/CMakeLists.txt:21-25 keeps the reference's scalar backend scalar).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define PAO_NEG_BIG (-3.0e38f)

/* ------------------------------------------------------------------------ */
/* decode: exact two-pass softmax, one (b, h) at a time                      */
/* ------------------------------------------------------------------------ */

/* One (b, h) row of cpu_reference (paged_attn_v1_hip.cpp:107-139).  `score`
 * is caller scratch of at least ctx floats. */
static void decode_row(float* out, const float* k, const float* v,
                       const float* q, const int32_t* bt, const int32_t* ctx,
                       int64_t b, int64_t h, int64_t H, int64_t HKV, int64_t D,
                       int64_t BS, int64_t MB, float scale, float* score) {
  const int64_t kv_h = h / (H / HKV);
  const int64_t n = ctx[b];
  float* o = out + (b * H + h) * D;
  if (n <= 0) {
    for (int64_t d = 0; d < D; ++d) o[d] = NAN;
    return;
  }
  const float* qr = q + (b * H + h) * D;
  float mx = PAO_NEG_BIG;
  for (int64_t j = 0; j < n; ++j) {
    const int64_t blk = bt[b * MB + j / BS], off = j % BS;
    const float* kr = k + ((blk * BS + off) * HKV + kv_h) * D;
    float dot = 0.0f;
    for (int64_t d = 0; d < D; ++d) dot += qr[d] * kr[d];
    score[j] = dot * scale;
    mx = score[j] > mx ? score[j] : mx;
  }
  float denom = 0.0f;
  for (int64_t j = 0; j < n; ++j) {
    score[j] = expf(score[j] - mx);
    denom += score[j];
  }
  for (int64_t d = 0; d < D; ++d) {
    float acc = 0.0f;
    for (int64_t j = 0; j < n; ++j) {
      const int64_t blk = bt[b * MB + j / BS], off = j % BS;
      acc += score[j] * v[((blk * BS + off) * HKV + kv_h) * D + d];
    }
    o[d] = acc / denom;
  }
}

typedef struct {
  float* out;
  const float *k, *v, *q;
  const int32_t *bt, *ctx;
  int64_t B, H, HKV, D, BS, MB;
  float scale;
  int64_t row_begin, row_end; /* flat (b, h) rows */
} decode_job;

static void* decode_worker(void* arg) {
  decode_job* j = (decode_job*)arg;
  float* score = (float*)malloc(sizeof(float) * (size_t)(j->MB * j->BS + 1));
  if (!score) return (void*)1;
  for (int64_t r = j->row_begin; r < j->row_end; ++r)
    decode_row(j->out, j->k, j->v, j->q, j->bt, j->ctx, r / j->H, r % j->H, j->H,
               j->HKV, j->D, j->BS, j->MB, j->scale, score);
  free(score);
  return NULL;
}

/* Paged decode.  q [B,H,D] f32; k,v [NB,BS,HKV,D] f32; bt [B,MB] i32;
 * ctx [B] i32; out [B,H,D] f32.  `threads` <= 1 runs the reference's single
 * thread; more threads split the (b, h) rows, each row computed exactly as
 * in the single-threaded loop, so results do not depend on `threads`.
 * Returns 0 on success. */
int pao_decode(float* out, const float* k, const float* v, const float* q,
               const int32_t* bt, const int32_t* ctx, int64_t B, int64_t H,
               int64_t HKV, int64_t D, int64_t BS, int64_t MB, float scale,
               int threads) {
  if (B < 0 || H <= 0 || HKV <= 0 || H % HKV || D <= 0 || BS <= 0 || MB < 0)
    return 1;
  const int64_t rows = B * H;
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if ((int64_t)threads > rows) threads = rows > 0 ? (int)rows : 1;
  decode_job jobs[256];
  pthread_t tids[256];
  for (int t = 0; t < threads; ++t) {
    decode_job j = {out, k, v, q, bt, ctx, B, H, HKV, D, BS, MB, scale,
                    rows * t / threads, rows * (t + 1) / threads};
    jobs[t] = j;
  }
  if (threads == 1) return decode_worker(&jobs[0]) ? 2 : 0;
  int rc = 0;
  for (int t = 0; t < threads; ++t)
    if (pthread_create(&tids[t], NULL, decode_worker, &jobs[t])) return 3;
  for (int t = 0; t < threads; ++t) {
    void* r = NULL;
    pthread_join(tids[t], &r);
    if (r) rc = 2;
  }
  return rc;
}

/* ------------------------------------------------------------------------ */
/* decode, split-KV formulation (v3): per-split online softmax + LSE merge   */
/* ------------------------------------------------------------------------ */

/* Scalar restatement of paged_attention_split_kernel (paged_attn_v3.cu:65-122)
 * followed by merge_splits_kernel (:139-165), in float, with the same chunking
 * chunk = ceil(ctx / S), the same -3e38 initial max and the same un-normalised
 * partials.  expf stands in for the kernel's __expf.  Returns 0 on success. */
int pao_decode_split(float* out, const float* k, const float* v, const float* q,
                     const int32_t* bt, const int32_t* ctx, int64_t B, int64_t H,
                     int64_t HKV, int64_t D, int64_t BS, int64_t MB, float scale,
                     int64_t S) {
  if (B < 0 || H <= 0 || HKV <= 0 || H % HKV || D <= 0 || BS <= 0 || S <= 0)
    return 1;
  float* pacc = (float*)malloc(sizeof(float) * (size_t)(S * D));
  float* pm = (float*)malloc(sizeof(float) * (size_t)S);
  float* pl = (float*)malloc(sizeof(float) * (size_t)S);
  if (!pacc || !pm || !pl) { free(pacc); free(pm); free(pl); return 2; }
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t h = 0; h < H; ++h) {
      const int64_t kv_h = h / (H / HKV);
      const int64_t n = ctx[b];
      const int64_t chunk = (n + S - 1) / S;
      const float* qr = q + (b * H + h) * D;
      for (int64_t s = 0; s < S; ++s) {
        const int64_t start = s * chunk;
        const int64_t end = start + chunk < n ? start + chunk : n;
        float m = PAO_NEG_BIG, l = 0.0f;
        float* acc = pacc + s * D;
        for (int64_t d = 0; d < D; ++d) acc[d] = 0.0f;
        for (int64_t j = start; j < end; ++j) {
          const int64_t blk = bt[b * MB + j / BS], off = j % BS;
          const int64_t base = ((blk * BS + off) * HKV + kv_h) * D;
          float dot = 0.0f;
          for (int64_t d = 0; d < D; ++d) dot += qr[d] * k[base + d];
          const float sc = dot * scale;
          const float m_new = m > sc ? m : sc;
          const float corr = expf(m - m_new);
          const float p = expf(sc - m_new);
          l = l * corr + p;
          for (int64_t d = 0; d < D; ++d) acc[d] = acc[d] * corr + p * v[base + d];
          m = m_new;
        }
        pm[s] = m;
        pl[s] = l;
      }
      float m_g = PAO_NEG_BIG;
      for (int64_t s = 0; s < S; ++s) m_g = pm[s] > m_g ? pm[s] : m_g;
      float l_g = 0.0f;
      float* o = out + (b * H + h) * D;
      for (int64_t d = 0; d < D; ++d) o[d] = 0.0f;
      for (int64_t s = 0; s < S; ++s) {
        const float w = expf(pm[s] - m_g);
        l_g += pl[s] * w;
        for (int64_t d = 0; d < D; ++d) o[d] += pacc[s * D + d] * w;
      }
      const float inv = 1.0f / l_g;
      for (int64_t d = 0; d < D; ++d) o[d] = o[d] * inv;
    }
  }
  free(pacc); free(pm); free(pl);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* causal chunked prefill                                                    */
/* ------------------------------------------------------------------------ */

typedef struct {
  float* out;
  const float *k, *v, *q;
  const int32_t *bt, *ctx;
  int64_t B, Sq, H, HKV, D, BS, MB;
  float scale;
  int64_t row_begin, row_end; /* flat (b, s, h) rows */
} prefill_job;

/* Query s of sequence b sits at absolute position ctx - Sq + s and attends to
 * keys [0, ctx - Sq + s] (paged_attn_prefill.cu:62-65); rows with no key
 * (end <= 0) are written as zeros (:70-74).  The softmax itself is
 * cpu_reference's two-pass form (paged_attn_v1_hip.cpp:111-138). */
static void* prefill_worker(void* arg) {
  prefill_job* J = (prefill_job*)arg;
  float* score = (float*)malloc(sizeof(float) * (size_t)(J->MB * J->BS + 1));
  if (!score) return (void*)1;
  for (int64_t r = J->row_begin; r < J->row_end; ++r) {
    const int64_t h = r % J->H;
    const int64_t s = (r / J->H) % J->Sq;
    const int64_t b = r / (J->H * J->Sq);
    const int64_t kv_h = h / (J->H / J->HKV);
    const int64_t end = (int64_t)J->ctx[b] - J->Sq + s + 1;
    float* o = J->out + ((b * J->Sq + s) * J->H + h) * J->D;
    if (end <= 0) {
      for (int64_t d = 0; d < J->D; ++d) o[d] = 0.0f;
      continue;
    }
    const float* qr = J->q + ((b * J->Sq + s) * J->H + h) * J->D;
    float mx = PAO_NEG_BIG;
    for (int64_t j = 0; j < end; ++j) {
      const int64_t blk = J->bt[b * J->MB + j / J->BS], off = j % J->BS;
      const float* kr = J->k + ((blk * J->BS + off) * J->HKV + kv_h) * J->D;
      float dot = 0.0f;
      for (int64_t d = 0; d < J->D; ++d) dot += qr[d] * kr[d];
      score[j] = dot * J->scale;
      mx = score[j] > mx ? score[j] : mx;
    }
    float denom = 0.0f;
    for (int64_t j = 0; j < end; ++j) {
      score[j] = expf(score[j] - mx);
      denom += score[j];
    }
    for (int64_t d = 0; d < J->D; ++d) {
      float acc = 0.0f;
      for (int64_t j = 0; j < end; ++j) {
        const int64_t blk = J->bt[b * J->MB + j / J->BS], off = j % J->BS;
        acc += score[j] * J->v[((blk * J->BS + off) * J->HKV + kv_h) * J->D + d];
      }
      o[d] = acc / denom;
    }
  }
  free(score);
  return NULL;
}

/* q, out [B,Sq,H,D] f32; k,v [NB,BS,HKV,D] f32.  ctx[b] must be <= MB*BS. */
int pao_prefill(float* out, const float* k, const float* v, const float* q,
                const int32_t* bt, const int32_t* ctx, int64_t B, int64_t Sq,
                int64_t H, int64_t HKV, int64_t D, int64_t BS, int64_t MB,
                float scale, int threads) {
  if (B < 0 || Sq < 0 || H <= 0 || HKV <= 0 || H % HKV || D <= 0 || BS <= 0)
    return 1;
  for (int64_t b = 0; b < B; ++b)
    if ((int64_t)ctx[b] > MB * BS) return 4;
  const int64_t rows = B * Sq * H;
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if ((int64_t)threads > rows) threads = rows > 0 ? (int)rows : 1;
  prefill_job jobs[256];
  pthread_t tids[256];
  for (int t = 0; t < threads; ++t) {
    prefill_job j = {out, k, v, q, bt, ctx, B, Sq, H, HKV, D, BS, MB, scale,
                     rows * t / threads, rows * (t + 1) / threads};
    jobs[t] = j;
  }
  if (threads == 1) return prefill_worker(&jobs[0]) ? 2 : 0;
  int rc = 0;
  for (int t = 0; t < threads; ++t)
    if (pthread_create(&tids[t], NULL, prefill_worker, &jobs[t])) return 3;
  for (int t = 0; t < threads; ++t) {
    void* r = NULL;
    pthread_join(tids[t], &r);
    if (r) rc = 2;
  }
  return rc;
}

/* ------------------------------------------------------------------------ */
/* split-count heuristic                                                     */
/* ------------------------------------------------------------------------ */

/* kernels/paged_attn_v3.cu:170-190: a chain-length target of 32 tokens per
 * split, a device-fill floor of 8 warps per SM, clamped to [1, 64]. */
int64_t pao_choose_num_splits(int64_t num_seqs, int64_t num_heads,
                              int64_t max_context, int64_t sms) {
  int64_t have = num_seqs * num_heads;
  if (have < 1) have = 1;
  int64_t by_chain = max_context / 32;
  if (by_chain < 1) by_chain = 1;
  int64_t fill = (sms * 8 + have - 1) / have;
  if (fill < 1) fill = 1;
  int64_t s = by_chain > fill ? by_chain : fill;
  if (s > 64) s = 64;
  if (s < 1) s = 1;
  return s;
}

/* ------------------------------------------------------------------------ */
/* scalar dot / scores / softmax (the CPU lane's scalar backend)             */
/* ------------------------------------------------------------------------ */

/* arm_cpu/src/scalar.cpp:9-15 */
float pao_dot(const float* a, const float* b, int64_t n) {
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) sum += a[i] * b[i];
  return sum;
}

/* arm_cpu/src/scalar.cpp:17-26 */
void pao_scores(const float* query, const float* keys, float* scores,
                int64_t tokens, int64_t head_dim) {
  for (int64_t t = 0; t < tokens; ++t)
    scores[t] = pao_dot(query, keys + t * head_dim, head_dim);
}

/* arm_cpu/src/scalar.cpp:28-46 */
void pao_softmax(float* scores, int64_t n) {
  if (n == 0) return;
  float mx = -INFINITY;
  for (int64_t i = 0; i < n; ++i) mx = scores[i] > mx ? scores[i] : mx;
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    scores[i] = expf(scores[i] - mx);
    sum += scores[i];
  }
  const float inv = 1.0f / sum;
  for (int64_t i = 0; i < n; ++i) scores[i] *= inv;
}
