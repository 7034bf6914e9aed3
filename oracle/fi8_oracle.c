/*
 * fi8_oracle.c -- CPU restatement of the reference's FlatI8 / FlatBinaryI8
 * exact-scan path. TEST INFRASTRUCTURE ONLY: used by tests/ as the parity
 * checker and by bench.py's CPU-baseline leg; the product never links it.
 *
 * Build (oracle/Makefile): gcc -O2 -ffp-contract=off -fno-fast-math -mavx2
 * -mpopcnt -fPIC -shared -pthread. Every float expression below is evaluated
 * in IEEE binary32 exactly as Go evaluates it on amd64 (SSE, round to nearest
 * even, no fused multiply-add).
 */
#define _GNU_SOURCE
#include "fi8_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------- */
/* Quantization: linalg/quant.go:43-71                                      */
/* ---------------------------------------------------------------------- */

/* Go's float64 -> int8 conversion on amd64 goes through CVTTSD2SL, whose
 * "integer indefinite" result for NaN (0x80000000) truncates to 0. Every
 * non-NaN value reaching here is already an integer in [-127, 127]. */
static int8_t go_f64_to_i8(double x) {
  if (x != x) return 0;
  return (int8_t)(int32_t)x;
}

float or_quantize_row(const float* row, int64_t d, int8_t* q, float zero_scale) {
  float maxAbs = 0.0f;
  for (int64_t i = 0; i < d; i++) { /* quant.go:44-52 */
    float v = row[i];
    if (v < 0) v = -v;
    if (v > maxAbs) maxAbs = v;
  }
  if (maxAbs == 0) { /* quant.go:53-58 */
    memset(q, 0, (size_t)d);
    return zero_scale;
  }
  float s = maxAbs / 127.0f; /* quant.go:59 (float32 divide) */
  float inv = 1.0f / s;      /* quant.go:60 (float32 divide) */
  for (int64_t j = 0; j < d; j++) { /* quant.go:61-69 */
    double x = round((double)(row[j] * inv)); /* math.Round: half away from 0 */
    if (x > 127) x = 127;
    else if (x < -127) x = -127;
    q[j] = go_f64_to_i8(x);
  }
  return s;
}

void or_quantize_rows(const float* v, int64_t n, int64_t d, int8_t* q,
                      float* scales, float zero_scale) {
  for (int64_t i = 0; i < n; i++) /* ann/flat_i8.go:96-107 */
    scales[i] = or_quantize_row(v + i * d, d, q + i * d, zero_scale);
}

/* ---------------------------------------------------------------------- */
/* int8 dot: linalg/quant.go:150, quant_i8_amd64.go:10-21, dot_amd64.s      */
/* ---------------------------------------------------------------------- */

int32_t or_dot_i8_scalar(const int8_t* a, const int8_t* b, int64_t d) {
  int32_t s = 0;
  for (int64_t k = 0; k < d; k++) s += (int32_t)a[k] * (int32_t)b[k];
  return s;
}

/* dotI8AVX2 (dot_amd64.s:323-387): sign-extend 16 bytes to int16
 * (VPMOVSXBW), pairwise multiply-add to int32 (VPMADDWD), four independent
 * accumulators over 64-byte iterations, then a 16-byte loop, then a
 * horizontal sum. n16 is a multiple of 16. */
__attribute__((target("avx2"))) static int32_t dot_i8_avx2(const int8_t* a,
                                                           const int8_t* b,
                                                           int64_t n16) {
  __m256i acc0 = _mm256_setzero_si256(), acc1 = acc0, acc2 = acc0, acc3 = acc0;
  int64_t i = 0;
  for (; i + 64 <= n16; i += 64) {
    __m256i a0 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + i)));
    __m256i b0 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + i)));
    acc0 = _mm256_add_epi32(acc0, _mm256_madd_epi16(a0, b0));
    __m256i a1 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + i + 16)));
    __m256i b1 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + i + 16)));
    acc1 = _mm256_add_epi32(acc1, _mm256_madd_epi16(a1, b1));
    __m256i a2 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + i + 32)));
    __m256i b2 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + i + 32)));
    acc2 = _mm256_add_epi32(acc2, _mm256_madd_epi16(a2, b2));
    __m256i a3 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + i + 48)));
    __m256i b3 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + i + 48)));
    acc3 = _mm256_add_epi32(acc3, _mm256_madd_epi16(a3, b3));
  }
  acc0 = _mm256_add_epi32(_mm256_add_epi32(acc0, acc1), _mm256_add_epi32(acc2, acc3));
  for (; i + 16 <= n16; i += 16) {
    __m256i a0 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + i)));
    __m256i b0 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + i)));
    acc0 = _mm256_add_epi32(acc0, _mm256_madd_epi16(a0, b0));
  }
  __m128i x = _mm_add_epi32(_mm256_castsi256_si128(acc0), _mm256_extracti128_si256(acc0, 1));
  x = _mm_hadd_epi32(x, x);
  x = _mm_hadd_epi32(x, x);
  return _mm_cvtsi128_si32(x);
}

static int g_has_avx2 = -1;

int32_t or_dot_i8(const int8_t* a, const int8_t* b, int64_t d) {
  if (g_has_avx2 < 0) g_has_avx2 = __builtin_cpu_supports("avx2") ? 1 : 0;
  if (!g_has_avx2 || d < 16) return or_dot_i8_scalar(a, b, d);
  int64_t n16 = d & ~(int64_t)15;
  int32_t s = dot_i8_avx2(a, b, n16);
  for (int64_t k = n16; k < d; k++) s += (int32_t)a[k] * (int32_t)b[k];
  return s;
}

/* ---------------------------------------------------------------------- */
/* W8A8 span + column fan-out: linalg/quant.go:248-298, linalg.go:208-233   */
/* ---------------------------------------------------------------------- */

typedef struct {
  const int8_t* aq;
  const float* ascales;
  int64_t M;
  const int8_t* bq;
  const float* bscales;
  int64_t N, d;
  float* dst;
  int64_t j0, j1;
} w8a8_job;

static void w8a8_span(const w8a8_job* jb) {
  for (int64_t j = jb->j0; j < jb->j1; j++) { /* quant.go:287-297 */
    const int8_t* bj = jb->bq + j * jb->d;
    float bScale = jb->bscales[j];
    for (int64_t i = 0; i < jb->M; i++) {
      if (jb->ascales[i] == 0) {
        jb->dst[i * jb->N + j] = 0;
        continue;
      }
      float f = (float)or_dot_i8(jb->aq + i * jb->d, bj, jb->d);
      f = f * jb->ascales[i];
      f = f * bScale;
      jb->dst[i * jb->N + j] = f;
    }
  }
}

static void* w8a8_thread(void* p) {
  w8a8_span((const w8a8_job*)p);
  return NULL;
}

void or_w8a8(const int8_t* aq, const float* ascales, int64_t M,
             const int8_t* bq, const float* bscales, int64_t N, int64_t d,
             float* dst, int nthreads) {
  w8a8_job base = {aq, ascales, M, bq, bscales, N, d, dst, 0, N};
  if (nthreads <= 1 || N < 2) {
    w8a8_span(&base);
    return;
  }
  int64_t workers = nthreads > N ? N : nthreads;
  int64_t chunk = (N + workers - 1) / workers; /* linalg.go:222-229 */
  if (chunk % 8) chunk += 8 - chunk % 8;
  int64_t nj = (N + chunk - 1) / chunk;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nj);
  w8a8_job* jobs = (w8a8_job*)malloc(sizeof(w8a8_job) * (size_t)nj);
  for (int64_t t = 0; t < nj; t++) {
    jobs[t] = base;
    jobs[t].j0 = t * chunk;
    jobs[t].j1 = (t + 1) * chunk < N ? (t + 1) * chunk : N;
    pthread_create(&th[t], NULL, w8a8_thread, &jobs[t]);
  }
  for (int64_t t = 0; t < nj; t++) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
}

/* ---------------------------------------------------------------------- */
/* topk.Selector: topk/topk.go:32-226; topk.Cmp/ItemCmp: topk/cmp.go:15-34  */
/* ---------------------------------------------------------------------- */

typedef struct {
  int64_t item;
  double score;
  uint64_t seq;
} scored;

typedef struct {
  int64_t k;
  uint64_t seq;
  int64_t len;
  scored* heap;
} selector;

static int heap_less(const scored* a, const scored* b) { /* topk.go:44-49 */
  if (a->score != b->score) return a->score < b->score;
  return a->seq > b->seq;
}

static void sift_down(scored* h, int64_t n, int64_t i) { /* topk.go:209-226 */
  for (;;) {
    int64_t l = 2 * i + 1, r = 2 * i + 2, s = i;
    if (l < n && heap_less(&h[l], &h[s])) s = l;
    if (r < n && heap_less(&h[r], &h[s])) s = r;
    if (s == i) return;
    scored t = h[i];
    h[i] = h[s];
    h[s] = t;
    i = s;
  }
}

static void sel_init(selector* s, int64_t k) {
  s->k = k;
  s->seq = 0;
  s->len = 0;
  s->heap = (scored*)malloc(sizeof(scored) * (size_t)(k > 0 ? k : 1));
}

static void sel_free(selector* s) { free(s->heap); }

static int sel_push(selector* s, int64_t item, double score) { /* topk.go:85-115 */
  if (s->k == 0) return 0;
  if (score != score) return 0;
  uint64_t seq = s->seq++;
  if (s->len < s->k) {
    int64_t i = s->len++;
    s->heap[i] = (scored){item, score, seq};
    while (i > 0) { /* siftUp, topk.go:194-203 */
      int64_t p = (i - 1) / 2;
      if (!heap_less(&s->heap[i], &s->heap[p])) break;
      scored t = s->heap[i];
      s->heap[i] = s->heap[p];
      s->heap[p] = t;
      i = p;
    }
    return 1;
  }
  if (score <= s->heap[0].score) return 0;
  s->heap[0] = (scored){item, score, seq};
  sift_down(s->heap, s->len, 0);
  return 1;
}

static double sel_threshold(const selector* s) { /* topk.go:137-149 */
  if (s->k == 0) return INFINITY;
  if (s->len < s->k) return -INFINITY;
  return s->heap[0].score;
}

/* Result (topk.go:171-186): repeated extract-min, filled back to front. */
static int64_t sel_result(const selector* s, int64_t* items, double* scores) {
  int64_t n = s->len;
  scored* tmp = (scored*)malloc(sizeof(scored) * (size_t)(n > 0 ? n : 1));
  memcpy(tmp, s->heap, sizeof(scored) * (size_t)n);
  int64_t len = n;
  for (int64_t i = n - 1; i >= 0; i--) {
    scored m = tmp[0];
    tmp[0] = tmp[len - 1];
    len--;
    sift_down(tmp, len, 0);
    items[i] = m.item;
    scores[i] = m.score;
  }
  free(tmp);
  return n;
}

typedef struct {
  int64_t id;
  double score;
} hit;

static int hit_cmp(const void* pa, const void* pb) { /* topk/cmp.go:15-26 */
  const hit* a = (const hit*)pa;
  const hit* b = (const hit*)pb;
  if (a->score > b->score) return -1;
  if (a->score < b->score) return 1;
  if (a->id < b->id) return -1;
  if (a->id > b->id) return 1;
  return 0;
}

static void sort_hits(int64_t* idx, double* score, int64_t n) {
  hit* h = (hit*)malloc(sizeof(hit) * (size_t)(n > 0 ? n : 1));
  for (int64_t i = 0; i < n; i++) h[i] = (hit){idx[i], score[i]};
  qsort(h, (size_t)n, sizeof(hit), hit_cmp);
  for (int64_t i = 0; i < n; i++) {
    idx[i] = h[i].id;
    score[i] = h[i].score;
  }
  free(h);
}

int64_t or_top_hits(const float* scores, int64_t n, int64_t k,
                    const uint8_t* keep, int64_t* out_idx, double* out_score) {
  if (k <= 0 || k >= n) { /* flat_i8.go:215-224: everything, sorted */
    int64_t c = 0;
    for (int64_t i = 0; i < n; i++)
      if (!keep || keep[i]) {
        out_idx[c] = i;
        out_score[c] = (double)scores[i];
        c++;
      }
    sort_hits(out_idx, out_score, c);
    return c;
  }
  selector sel; /* flat_i8.go:226-245 */
  sel_init(&sel, k);
  double th = sel_threshold(&sel);
  for (int64_t i = 0; i < n; i++) {
    double s = (double)scores[i];
    if (s > th && (!keep || keep[i])) {
      sel_push(&sel, i, s);
      th = sel_threshold(&sel);
    }
  }
  int64_t c = sel_result(&sel, out_idx, out_score);
  sel_free(&sel);
  sort_hits(out_idx, out_score, c);
  return c;
}

int64_t or_flat_i8_query(const int8_t* bq, const float* scales, int64_t n,
                         int64_t d, const float* q, int64_t k,
                         const uint8_t* keep, int64_t* out_idx,
                         double* out_score, int nthreads) {
  if (n == 0) return -1; /* flat_i8.go:151-153 */
  int8_t* aq = (int8_t*)malloc((size_t)(d > 0 ? d : 1));
  float as = or_quantize_row(q, d, aq, 0.0f); /* quant.go:171 via :204-207 */
  float* dst = (float*)malloc(sizeof(float) * (size_t)n);
  or_w8a8(aq, &as, 1, bq, scales, n, d, dst, nthreads);
  int64_t c = or_top_hits(dst, n, k, keep, out_idx, out_score);
  free(aq);
  free(dst);
  return c;
}

int64_t or_merge_hits(const int64_t* idx, const double* score, int64_t total,
                      int64_t k, int64_t* out_idx, double* out_score) {
  int64_t* ti = (int64_t*)malloc(sizeof(int64_t) * (size_t)(total > 0 ? total : 1));
  double* ts = (double*)malloc(sizeof(double) * (size_t)(total > 0 ? total : 1));
  memcpy(ti, idx, sizeof(int64_t) * (size_t)total);
  memcpy(ts, score, sizeof(double) * (size_t)total);
  sort_hits(ti, ts, total); /* backend.go:270-271 */
  int64_t c = total > k ? k : total; /* backend.go:272-274 */
  memcpy(out_idx, ti, sizeof(int64_t) * (size_t)c);
  memcpy(out_score, ts, sizeof(double) * (size_t)c);
  free(ti);
  free(ts);
  return c;
}

/* ---------------------------------------------------------------------- */
/* Binary prefilter: ann/flat_binary_prefilter.go, linalg/hamming.go        */
/* ---------------------------------------------------------------------- */

int64_t or_center(const float* v, int64_t n, int64_t d, const uint8_t* valid,
                  float* center) {
  double* acc = (double*)calloc((size_t)(d > 0 ? d : 1), sizeof(double));
  int64_t used = 0;
  for (int64_t r = 0; r < n; r++) { /* prefilter.go:70-78 */
    if (valid && !valid[r]) continue;
    used++;
    for (int64_t i = 0; i < d; i++) acc[i] += (double)v[r * d + i];
  }
  if (used > 0) /* prefilter.go:79-84 */
    for (int64_t i = 0; i < d; i++) center[i] = (float)(acc[i] / (double)used);
  free(acc);
  return used;
}

void or_pack_row(const float* v, const float* center, int64_t d, uint64_t* dst) {
  int64_t w = (d + 63) / 64; /* hamming.go:28-36 */
  memset(dst, 0, sizeof(uint64_t) * (size_t)w);
  for (int64_t i = 0; i < d; i++) {
    float x = center ? v[i] - center[i] : v[i]; /* prefilter.go:100-108 */
    if (x >= 0) dst[i >> 6] |= (uint64_t)1 << (i & 63);
  }
}

void or_pack_codes(const float* v, const float* center, int64_t n, int64_t d,
                   const uint8_t* valid, uint64_t* codes) {
  int64_t w = (d + 63) / 64;
  memset(codes, 0, sizeof(uint64_t) * (size_t)(n * w));
  for (int64_t r = 0; r < n; r++) { /* prefilter.go:87-95 */
    if (valid && !valid[r]) continue;
    or_pack_row(v + r * d, center, d, codes + r * w);
  }
}

void or_hamming_rows(const uint64_t* q, const uint64_t* codes, int64_t words,
                     int64_t n, uint16_t* dst) {
  for (int64_t i = 0; i < n; i++) { /* hamming.go:64-73 */
    int s = 0;
    for (int64_t j = 0; j < words; j++) s += __builtin_popcountll(codes[i * words + j] ^ q[j]);
    dst[i] = (uint16_t)s;
  }
}

typedef struct {
  const uint64_t* qc;
  const uint64_t* codes;
  int64_t words, lo, hi, nb;
  uint16_t* dists;
  int64_t* hist;
} hist_job;

/* scanHist (prefilter.go:207-216) over rows [lo, hi) in 1024-row blocks. */
static void hist_span(const hist_job* j) {
  for (int64_t base = j->lo; base < j->hi; base += 1024) {
    int64_t end = base + 1024 < j->hi ? base + 1024 : j->hi;
    or_hamming_rows(j->qc, j->codes + base * j->words, j->words, end - base, j->dists + base);
    for (int64_t i = base; i < end; i++) j->hist[j->dists[i]]++;
  }
}

static void* hist_thread(void* arg) {
  hist_span((const hist_job*)arg);
  return NULL;
}

int64_t or_prefilter_hist_mt(const uint64_t* qc, const uint64_t* codes, int64_t n,
                             int64_t dim, int64_t cand, int32_t* ids_out, int nthreads) {
  int64_t words = (dim + 63) / 64;
  int64_t nb = dim + 1;
  uint16_t* dists = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(n > 0 ? n : 1));
  /* the worker split of prefilter.go:147-178: binQueryWorkers (:328-335,
   * one worker below 2^17 scanned words, else one per CPU) workers, each
   * scanning a contiguous row range into its own histogram; the histograms
   * are summed. Results do not depend on the split. */
  int64_t workers = (nthreads < 1 || n < 2 || n * words < (1 << 17)) ? 1 : (nthreads < n ? nthreads : n);
  int64_t per = (n + workers - 1) / workers;
  int64_t* hist = (int64_t*)calloc((size_t)(nb * workers), sizeof(int64_t));
  hist_job* jobs = (hist_job*)malloc(sizeof(hist_job) * (size_t)workers);
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)workers);
  for (int64_t w = 0; w < workers; w++) {
    int64_t lo = w * per, hi = lo + per < n ? lo + per : n;
    hist_job jb = {qc, codes, words, lo < n ? lo : n, hi, nb, dists, hist + w * nb};
    jobs[w] = jb;
    if (workers > 1) pthread_create(&th[w], NULL, hist_thread, &jobs[w]);
  }
  if (workers == 1) hist_span(&jobs[0]);
  else
    for (int64_t w = 0; w < workers; w++) pthread_join(th[w], NULL);
  for (int64_t w = 1; w < workers; w++)
    for (int64_t b = 0; b < nb; b++) hist[b] += hist[w * nb + b];
  free(jobs);
  free(th);
  int64_t cum = 0, t = 0; /* prefilter.go:182-189 */
  for (; t < nb; t++) {
    if (cum + hist[t] >= cand) break;
    cum += hist[t];
  }
  int64_t budget = cand - cum;
  int64_t c = 0; /* prefilter.go:191-200 */
  for (int64_t i = 0; i < n; i++) {
    int64_t dd = dists[i];
    if (dd < t) ids_out[c++] = (int32_t)i;
    else if (dd == t && budget > 0) {
      ids_out[c++] = (int32_t)i;
      budget--;
    }
  }
  free(dists);
  free(hist);
  return c;
}

int64_t or_prefilter_hist(const uint64_t* qc, const uint64_t* codes, int64_t n,
                          int64_t dim, int64_t cand, int32_t* ids_out) {
  return or_prefilter_hist_mt(qc, codes, n, dim, cand, ids_out, 1);
}

static int cmp_i32(const void* a, const void* b) {
  int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
  return (x > y) - (x < y);
}

int64_t or_prefilter_heap(const uint64_t* qc, const uint64_t* codes, int64_t n,
                          int64_t dim, int64_t cand, const uint8_t* keep,
                          int nshards, int32_t* ids_out) {
  int64_t words = (dim + 63) / 64;
  int64_t workers = nshards < 1 ? 1 : nshards;
  int64_t per = (n + workers - 1) / workers; /* prefilter.go:235 */
  int64_t cap = workers * (cand > 0 ? cand : 1);
  int64_t* mi = (int64_t*)malloc(sizeof(int64_t) * (size_t)cap);
  double* ms = (double*)malloc(sizeof(double) * (size_t)cap);
  int64_t nm = 0;
  uint16_t dist[1024];
  for (int64_t w = 0; w < workers; w++) {
    int64_t lo = w * per;
    if (lo >= n) break;
    int64_t hi = lo + per < n ? lo + per : n;
    selector sel; /* scanShard, prefilter.go:272-292 */
    sel_init(&sel, cand);
    double th = sel_threshold(&sel);
    for (int64_t base = lo; base < hi; base += 1024) {
      int64_t end = base + 1024 < hi ? base + 1024 : hi;
      or_hamming_rows(qc, codes + base * words, words, end - base, dist);
      for (int64_t j = 0; j < end - base; j++) {
        double s = -(double)dist[j];
        if (s > th && (!keep || keep[base + j])) {
          sel_push(&sel, base + j, s);
          th = sel_threshold(&sel);
        }
      }
    }
    nm += sel_result(&sel, mi + nm, ms + nm);
    sel_free(&sel);
  }
  sort_hits(mi, ms, nm); /* finishCandidates, prefilter.go:296-313 */
  int64_t c = nm > cand ? cand : nm;
  for (int64_t i = 0; i < c; i++) ids_out[i] = (int32_t)mi[i];
  qsort(ids_out, (size_t)c, sizeof(int32_t), cmp_i32);
  free(mi);
  free(ms);
  return c;
}

int64_t or_flat_binary_i8_query(const uint64_t* codes, const float* center,
                                int64_t words, const int8_t* bq,
                                const float* scales, int64_t n, int64_t d,
                                int64_t over, const float* q, int64_t k,
                                const uint8_t* keep, int64_t* out_idx,
                                double* out_score, int nthreads) {
  if (n == 0) return -1; /* flat_binary_i8.go:87-89 */
  if (over < 1) over = 1; /* prefilter.go:58 */
  int64_t cand;
  int ovf = __builtin_mul_overflow(k, over, &cand);
  if (k <= 0 || k >= n || ovf || cand >= n || cand < 0) /* :95-97 */
    return or_flat_i8_query(bq, scales, n, d, q, k, keep, out_idx, out_score, nthreads);
  uint64_t* qc = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)words);
  or_pack_row(q, center, d, qc); /* :101-103 */
  int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * (size_t)cand);
  int64_t nid = keep ? or_prefilter_heap(qc, codes, n, d, cand, keep, 1, ids)
                     : or_prefilter_hist_mt(qc, codes, n, d, cand, ids, nthreads);
  /* rerank (:122-153): gather in id order, one W8A8 call, topk in id order. */
  int8_t* g = (int8_t*)malloc((size_t)(nid * d > 0 ? nid * d : 1));
  float* gs = (float*)malloc(sizeof(float) * (size_t)(nid > 0 ? nid : 1));
  for (int64_t i = 0; i < nid; i++) {
    memcpy(g + i * d, bq + (int64_t)ids[i] * d, (size_t)d);
    gs[i] = scales[ids[i]];
  }
  int8_t* aq = (int8_t*)malloc((size_t)(d > 0 ? d : 1));
  float as = or_quantize_row(q, d, aq, 0.0f);
  float* dst = (float*)malloc(sizeof(float) * (size_t)(nid > 0 ? nid : 1));
  or_w8a8(aq, &as, 1, g, gs, nid, d, dst, nthreads);
  selector sel;
  sel_init(&sel, k);
  double th = sel_threshold(&sel);
  for (int64_t i = 0; i < nid; i++) {
    double s = (double)dst[i];
    if (s > th) {
      sel_push(&sel, ids[i], s);
      th = sel_threshold(&sel);
    }
  }
  int64_t c = sel_result(&sel, out_idx, out_score);
  sel_free(&sel);
  sort_hits(out_idx, out_score, c);
  free(qc);
  free(ids);
  free(g);
  free(gs);
  free(aq);
  free(dst);
  return c;
}
