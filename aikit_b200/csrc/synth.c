/*
 * synth.c -- seeded synthetic corpora for tests and benchmarks (host only).
 *
 * The reference measures on Model2Vec embeddings that are not available here;
 * these generators produce the shapes and value distributions the benchmark
 * configurations name instead. Every value is a pure function of
 * (seed, stream, row, column) through a counter-based hash, so any row range
 * can be regenerated independently and the output does not depend on the
 * thread count. The GPU never generates data: both the device and the CPU
 * oracle consume these host-made codes.
 *
 *   hash     splitmix64 finalizer chained over (seed, stream, counter)
 *   normal   inverse-CDF table: a 64-bit hash of (seed, stream, row, j/4)
 *            supplies four 16-bit uniforms; element j takes lane j%4 and maps
 *            it through a 65536-entry table of standard-normal quantiles
 *            Phi^-1((i + 0.5) / 65536), built once from Acklam's rational
 *            approximation refined by one Halley step on erfc
 *   unit     v_j = float32(z_j); s = sum(float64(v_j)^2);
 *            v *= float32(1/sqrt(s))  (the normalisation the reference's GPU
 *            tests use, gpu/anncuda/backend_test.go:20-36)
 *   mixture  centre c = N(0,1) row of the centre stream; cluster of a row =
 *            hash % nclusters; v_j = c_j + sigma*float32(z_j) in float32, then
 *            normalised as above
 *   ties     codes uniform over {-2..2}, scale fixed at float32(1/127)
 *
 * Corpus rows are quantized with QuantizeRowInt8's arithmetic
 * (linalg/quant.go:43-71, all-zero row -> scale 1), as NewFlatI8 does.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static inline uint64_t hash3(uint64_t seed, uint64_t stream, uint64_t ctr) {
  return mix64(mix64(mix64(seed) ^ stream) ^ ctr);
}


static float g_qtab[65536];
static pthread_once_t g_qtab_once = PTHREAD_ONCE_INIT;

/* Acklam's inverse-normal rational approximation plus one Halley step. */
static double inv_norm(double p) {
  static const double a[] = {-3.969683028665376e+01, 2.209460984245205e+02, -2.759285104469687e+02,
                             1.383577518672690e+02, -3.066479806614716e+01, 2.506628277459239e+00};
  static const double b[] = {-5.447609879822406e+01, 1.615858368580409e+02, -1.556989798598866e+02,
                             6.680131188771972e+01, -1.328068155288572e+01};
  static const double c[] = {-7.784894002430293e-03, -3.223964580411365e-01, -2.400758277161838e+00,
                             -2.549732539343734e+00, 4.374664141464968e+00, 2.938163982698783e+00};
  static const double dd[] = {7.784695709041462e-03, 3.224671290700398e-01, 2.445134137142996e+00,
                              3.754408661907416e+00};
  const double plow = 0.02425, phigh = 1 - plow;
  double x;
  if (p < plow) {
    const double q = sqrt(-2 * log(p));
    x = (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
        ((((dd[0] * q + dd[1]) * q + dd[2]) * q + dd[3]) * q + 1);
  } else if (p <= phigh) {
    const double q = p - 0.5, r = q * q;
    x = (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q /
        (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1);
  } else {
    const double q = sqrt(-2 * log(1 - p));
    x = -(((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
        ((((dd[0] * q + dd[1]) * q + dd[2]) * q + dd[3]) * q + 1);
  }
  const double e = 0.5 * erfc(-x / sqrt(2.0)) - p;
  const double u = e * sqrt(2 * 3.14159265358979323846) * exp(x * x / 2);
  return x - u / (1 + x * u / 2);
}

static void build_qtab(void) {
  for (int i = 0; i < 65536; i++) g_qtab[i] = (float)inv_norm((i + 0.5) / 65536.0);
}

/* Fill v[0..d) with standard normals for `row` of a stream. */
static void normal_row(uint64_t seed, uint64_t stream, int64_t row, int64_t d, float* v) {
  pthread_once(&g_qtab_once, build_qtab);
  const uint64_t per_row = (uint64_t)((d + 3) / 4);
  for (int64_t j0 = 0; j0 < d; j0 += 4) {
    const uint64_t h = hash3(seed, stream, (uint64_t)row * per_row + (uint64_t)(j0 / 4));
    for (int64_t l = 0; l < 4 && j0 + l < d; l++) v[j0 + l] = g_qtab[(h >> (16 * l)) & 0xFFFFu];
  }
}

static void normalize(float* v, int64_t d) {
  double s = 0.0;
  for (int64_t j = 0; j < d; j++) s += (double)v[j] * (double)v[j];
  if (s == 0.0) return;
  const float inv = (float)(1.0 / sqrt(s));
  for (int64_t j = 0; j < d; j++) v[j] *= inv;
}

float syn_quantize_row(const float* row, int64_t d, int8_t* q, float zero_scale) {
  float maxAbs = 0.0f;
  for (int64_t i = 0; i < d; i++) {
    float v = row[i];
    if (v < 0) v = -v;
    if (v > maxAbs) maxAbs = v;
  }
  if (maxAbs == 0) {
    memset(q, 0, (size_t)d);
    return zero_scale;
  }
  const float s = maxAbs / 127.0f;
  const float inv = 1.0f / s;
  for (int64_t j = 0; j < d; j++) {
    double x = round((double)(row[j] * inv));
    if (x > 127) x = 127;
    else if (x < -127) x = -127;
    q[j] = (x != x) ? 0 : (int8_t)(int32_t)x;
  }
  return s;
}

enum { KIND_UNIT = 0, KIND_MIXTURE = 1, KIND_TIES = 2 };

typedef struct {
  int kind;
  uint64_t seed, stream;
  const float* centers;
  int64_t ncl;
  float sigma;
  int64_t row0, r0, r1, d;
  float* out_f;     /* optional float rows */
  int8_t* out_q;    /* optional codes */
  float* out_s;     /* optional scales */
  const float* center;  /* sign codes: subtracted before the sign test (may be NULL) */
  uint64_t* out_bits;   /* optional packed sign codes, ceil(d/64) words per row */
  double* out_sum;      /* optional column sums, one d-vector per 4096-row block */
} job_t;

enum { SUM_BLOCK = 4096 };

static void gen_row(const job_t* jb, int64_t row, float* v) {
  const int64_t d = jb->d;
  if (jb->kind == KIND_TIES) {
    for (int64_t j = 0; j < d; j++) {
      const uint64_t h = hash3(jb->seed, jb->stream, (uint64_t)row * (uint64_t)d + (uint64_t)j);
      v[j] = (float)((int64_t)(h % 5u) - 2);
    }
    return;
  }
  if (jb->kind == KIND_MIXTURE) {
    const uint64_t c = hash3(jb->seed, jb->stream ^ 0xC1u, (uint64_t)row) % (uint64_t)jb->ncl;
    const float* ctr = jb->centers + c * (uint64_t)d;
    normal_row(jb->seed, jb->stream, row, d, v);
    for (int64_t j = 0; j < d; j++) v[j] = ctr[j] + jb->sigma * v[j];
  } else {
    normal_row(jb->seed, jb->stream, row, d, v);
  }
  normalize(v, d);
}

static void* run_job(void* p) {
  const job_t* jb = (const job_t*)p;
  float* tmp = (float*)malloc(sizeof(float) * (size_t)(jb->d > 0 ? jb->d : 1));
  const int64_t words = (jb->d + 63) / 64;
  for (int64_t r = jb->r0; r < jb->r1; r++) {
    const int64_t row = jb->row0 + r;
    float* v = jb->out_f ? jb->out_f + r * jb->d : tmp;
    gen_row(jb, row, v);
    if (jb->out_sum) {
      double* acc = jb->out_sum + (r / SUM_BLOCK) * jb->d;
      for (int64_t j = 0; j < jb->d; j++) acc[j] += (double)v[j];
    }
    if (jb->out_bits) {
      /* PackSignBitsRow of v - center (linalg/hamming.go:28-37) */
      uint64_t* w = jb->out_bits + r * words;
      memset(w, 0, sizeof(uint64_t) * (size_t)words);
      for (int64_t j = 0; j < jb->d; j++) {
        const float x = jb->center ? v[j] - jb->center[j] : v[j];
        if (x >= 0.0f) w[j >> 6] |= 1ull << (j & 63);
      }
    }
    if (jb->out_q) {
      if (jb->kind == KIND_TIES) {
        for (int64_t j = 0; j < jb->d; j++) jb->out_q[r * jb->d + j] = (int8_t)v[j];
        jb->out_s[r] = 1.0f / 127.0f;
      } else {
        jb->out_s[r] = syn_quantize_row(v, jb->d, jb->out_q + r * jb->d, 1.0f);
      }
    }
  }
  free(tmp);
  return NULL;
}

static void run_parallel(job_t base, int64_t nrows, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > nrows) nthreads = (int)(nrows > 0 ? nrows : 1);
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
  job_t* jobs = (job_t*)malloc(sizeof(job_t) * (size_t)nthreads);
  int64_t per = (nrows + nthreads - 1) / nthreads;
  if (base.out_sum) per = (per + SUM_BLOCK - 1) / SUM_BLOCK * SUM_BLOCK;  /* a block never spans threads */
  int started = 0;
  for (int t = 0; t < nthreads; t++) {
    jobs[t] = base;
    jobs[t].r0 = t * per;
    jobs[t].r1 = (t + 1) * per < nrows ? (t + 1) * per : nrows;
    if (jobs[t].r0 >= jobs[t].r1) break;
    pthread_create(&th[t], NULL, run_job, &jobs[t]);
    started++;
  }
  for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
}

/* N(0,1) rows (no normalisation), e.g. mixture centres. */
void syn_normal_rows(uint64_t seed, uint64_t stream, int64_t row0, int64_t nrows, int64_t d, float* out) {
  for (int64_t r = 0; r < nrows; r++) normal_row(seed, stream, row0 + r, d, out + r * d);
}

/* kind: 0 unit N(0,1), 1 mixture, 2 ties. Any of out_f / (out_q, out_s) may be
 * NULL; rows [row0, row0+nrows) of the stream are produced. */
void syn_rows(int kind, uint64_t seed, uint64_t stream, const float* centers, int64_t ncl, float sigma,
              int64_t row0, int64_t nrows, int64_t d, float* out_f, int8_t* out_q, float* out_s,
              int nthreads) {
  job_t base;
  memset(&base, 0, sizeof(base));
  base.kind = kind;
  base.seed = seed;
  base.stream = stream;
  base.centers = centers;
  base.ncl = ncl > 0 ? ncl : 1;
  base.sigma = sigma;
  base.row0 = row0;
  base.d = d;
  base.out_f = out_f;
  base.out_q = out_q;
  base.out_s = out_s;
  run_parallel(base, nrows, nthreads);
}

/* Column sums over rows [row0, row0+nrows) in float64, in the order: rows
 * summed within 4096-row blocks, then the blocks in row order. The result does
 * not depend on the thread count. out_sum [d]. */
void syn_column_sums(int kind, uint64_t seed, uint64_t stream, const float* centers, int64_t ncl, float sigma,
                     int64_t row0, int64_t nrows, int64_t d, double* out_sum, int nthreads) {
  const int64_t nblk = (nrows + SUM_BLOCK - 1) / SUM_BLOCK;
  double* part = (double*)calloc((size_t)(nblk > 0 ? nblk : 1) * (size_t)d, sizeof(double));
  job_t base;
  memset(&base, 0, sizeof(base));
  base.kind = kind;
  base.seed = seed;
  base.stream = stream;
  base.centers = centers;
  base.ncl = ncl > 0 ? ncl : 1;
  base.sigma = sigma;
  base.row0 = row0;
  base.d = d;
  base.out_sum = part;
  run_parallel(base, nrows, nthreads);
  for (int64_t j = 0; j < d; j++) out_sum[j] = 0.0;
  for (int64_t b = 0; b < nblk; b++)
    for (int64_t j = 0; j < d; j++) out_sum[j] += part[b * d + j];
  free(part);
}

/* Rows [row0, row0+nrows) as a FlatBinaryI8 corpus: packed sign codes of
 * (v - center) (center may be NULL) into out_bits [nrows][ceil(d/64)] and, if
 * out_q is given, the QuantizeRowInt8 codes and scales. */
void syn_binary_rows(int kind, uint64_t seed, uint64_t stream, const float* centers, int64_t ncl, float sigma,
                     int64_t row0, int64_t nrows, int64_t d, const float* center, uint64_t* out_bits,
                     int8_t* out_q, float* out_s, int nthreads) {
  job_t base;
  memset(&base, 0, sizeof(base));
  base.kind = kind;
  base.seed = seed;
  base.stream = stream;
  base.centers = centers;
  base.ncl = ncl > 0 ? ncl : 1;
  base.sigma = sigma;
  base.row0 = row0;
  base.d = d;
  base.center = center;
  base.out_bits = out_bits;
  base.out_q = out_q;
  base.out_s = out_s;
  run_parallel(base, nrows, nthreads);
}
