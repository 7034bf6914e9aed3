// fi8_api.cu -- the C ABI (include/fi8.h): device contexts, device-resident
// FlatI8 shards, and the Score / ScoreBatch / TopKBatch entry points that the
// reference's ann.Backend seam calls (ann/backend.go:16-55).
//
// Error behaviour follows gpu/anncuda/backend.go: shape errors and device
// failures are returned, never panicked; TopKBatch declines k <= 0 and k >= n
// (backend.go:577). Unlike the reference it does not decline small n (its
// topkMinN = 50_000, backend.go:305, is a launch-cost crossover of a two-kernel
// design; here scoring and selection are one launch).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/fi8.h"
#include "fi8_binary.cuh"
#include "fi8_build.cuh"
#include "fi8_device.cuh"
#include "fi8_gemm.cuh"
#include "fi8_scan.cuh"
#include "fi8_stage.h"

using namespace fi8;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  const int code = (e == cudaErrorMemoryAllocation) ? FI8_ERR_OOM : FI8_ERR_CUDA;
  return fail(code, "%s: %s", what, cudaGetErrorString(e));
}

#define FI8_CUDA(call, what)                      \
  do {                                            \
    cudaError_t e_ = (call);                      \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

template <typename T>
int ensure_device(T** p, size_t* cap, size_t need, const char* what) {
  if (*cap >= need && *p) return FI8_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  const size_t n = std::max<size_t>(need, 1);
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T));
  if (e != cudaSuccess) {
    *p = nullptr;
    return cuda_fail(e, what);
  }
  *cap = n;
  return FI8_OK;
}

template <typename T>
int ensure_host(T** p, size_t* cap, size_t need, const char* what) {
  if (*cap >= need && *p) return FI8_OK;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  const size_t n = std::max<size_t>(need, 1);
  cudaError_t e = cudaMallocHost(reinterpret_cast<void**>(p), n * sizeof(T));
  if (e != cudaSuccess) {
    *p = nullptr;
    return cuda_fail(e, what);
  }
  *cap = n;
  return FI8_OK;
}

// Queries handled per scan launch in the multi-query (one pass per query)
// form; bounds the per-launch scratch.
constexpr int32_t kScanMaxM = 64;
constexpr int64_t kRowAlign = 256;  // n is padded to a multiple of this

}  // namespace

struct fi8_ctx {
  int device = 0;
  int sm_count = 0;
};

struct fi8_index {
  fi8_ctx* ctx = nullptr;
  int device = 0;
  int sm_count = 0;
  int64_t n = 0, n_alloc = 0;
  int32_t dim = 0, dpad = 0;
  uint32_t id_base = 0;
  int8_t* d_codes = nullptr;
  float* d_scales = nullptr;
  cudaStream_t stream = nullptr;
  std::mutex mu;

  // top-K scan scratch, sized for (scr_M queries, scr_k, scr_G CTAs)
  unsigned long long* d_gthr = nullptr;
  size_t gthr_cap = 0;
  unsigned int* d_counter = nullptr;
  size_t counter_cap = 0;
  unsigned int* d_counter2 = nullptr;
  size_t counter2_cap = 0;
  uint64_t* d_lvl1 = nullptr;
  size_t lvl1_cap = 0;
  uint64_t* d_lvl2 = nullptr;
  size_t lvl2_cap = 0;
  unsigned int* d_err = nullptr;
  unsigned int* h_err = nullptr;
  // the batched path's redo gate: set (on the device) when a batch's select
  // dropped candidates, which opens the gated exact redo launched after it
  unsigned int* d_redo = nullptr;

  // staging for the host-pointer entry points
  float* d_q = nullptr;
  size_t d_q_cap = 0;
  uint64_t* d_keys = nullptr;
  size_t d_keys_cap = 0;
  float* d_scores = nullptr;
  size_t d_scores_cap = 0;
  uint64_t* h_keys = nullptr;
  size_t h_keys_cap = 0;

  // batched (tcgen05 GEMM) path
  CUtensorMap tmB;       // corpus codes [n_alloc][dpad], 256-row boxes
  bool has_tmB = false;
  CUtensorMap tmB2;      // the same rows in 128-row boxes (a CTA pair's halves)
  bool has_tmB2 = false;
  int8_t* d_A = nullptr;  // quantized queries [Mpad][dpad]
  size_t A_cap = 0;
  CUtensorMap tmA;       // over d_A, rebuilt when d_A moves
  const int8_t* tmA_base = nullptr;
  int64_t tmA_rows = 0;
  int32_t tmA_box = 0;   // query tile rows the map's box was built for
  float* d_qscale = nullptr;
  size_t qscale_cap = 0;
  unsigned long long* d_thr = nullptr;
  size_t thr_cap = 0;
  unsigned int* d_cnt = nullptr;
  size_t cnt_cap = 0;
  uint64_t* d_cand = nullptr;
  size_t cand_cap = 0;
  uint64_t* d_topk = nullptr;
  size_t topk_cap = 0;
  int32_t gemm_min_batch = 2;  // batches of at least this many queries use the GEMM path
  int32_t gemm_ctas = 0;       // cap on the GEMM's persistent CTAs (0: one per SM)
  int32_t gemm_pair = 0;       // batches of more than 128 queries on CTA pairs (FI8_OPT_GEMM_PAIR)
  int32_t last_launches = 0;   // kernels launched by the last query call

  // incremental uploads (fi8_index_upload_rows): the pinned double buffer,
  // held from the first upload until fi8_index_upload_finish or destroy
  PinnedStager* up_stage = nullptr;

  // keep filter of the call in progress (QueryFilter), null when none
  const uint64_t* cur_keep = nullptr;
  int64_t cur_keep_nbits = 0;
  uint64_t* d_keep = nullptr;  // device copy of a host bitmap
  size_t keep_cap = 0;

  // optional per-launch timing (FI8_OPT_KERNEL_TIMING)
  struct TimedLaunch {
    int kind;
    cudaEvent_t e0, e1;
    double bytes;
  };
  bool timing = false;
  std::vector<TimedLaunch> timed;
  std::vector<cudaEvent_t> event_pool;
};

namespace {

cudaEvent_t take_event(fi8_index* x) {
  cudaEvent_t e = nullptr;
  if (!x->event_pool.empty()) {
    e = x->event_pool.back();
    x->event_pool.pop_back();
  } else if (cudaEventCreate(&e) != cudaSuccess) {
    e = nullptr;
  }
  return e;
}

// Bracket one kernel launch with events when timing is on. begin() returns the
// start event (or null); end() records the stop event and files the launch.
cudaEvent_t timer_begin(fi8_index* x, cudaStream_t st) {
  if (!x->timing) return nullptr;
  cudaEvent_t e = take_event(x);
  if (e) cudaEventRecord(e, st);
  return e;
}

void timer_end(fi8_index* x, cudaStream_t st, cudaEvent_t e0, int kind, double bytes) {
  if (!e0) return;
  cudaEvent_t e1 = take_event(x);
  if (!e1) {
    x->event_pool.push_back(e0);
    return;
  }
  cudaEventRecord(e1, st);
  x->timed.push_back(fi8_index::TimedLaunch{kind, e0, e1, bytes});
}

}  // namespace

extern "C" {

const char* fi8_last_error(void) { return g_last_error.c_str(); }

int fi8_device_count(int* out) {
  if (!out) return fail(FI8_ERR_ARG, "fi8_device_count: null out");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    *out = 0;
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  *out = n;
  return FI8_OK;
}

int fi8_ctx_create(int device, fi8_ctx** out) {
  if (!out) return fail(FI8_ERR_ARG, "fi8_ctx_create: null out");
  *out = nullptr;
  int ndev = 0;
  FI8_CUDA(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
  if (device < 0 || device >= ndev) return fail(FI8_ERR_ARG, "fi8_ctx_create: device %d of %d", device, ndev);
  DeviceGuard g(device);
  cudaDeviceProp prop;
  FI8_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10) return fail(FI8_ERR_DECLINED, "fi8: device %d is sm_%d%d, this build targets sm_100a", device, prop.major, prop.minor);
  fi8_ctx* c = new (std::nothrow) fi8_ctx;
  if (!c) return fail(FI8_ERR_OOM, "fi8_ctx_create: host allocation");
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  *out = c;
  return FI8_OK;
}

int fi8_ctx_destroy(fi8_ctx* ctx) {
  delete ctx;
  return FI8_OK;
}

int fi8_probe_tensor_i8(fi8_ctx* ctx, int64_t iters, double* ops_per_s, double* ms) {
  if (!ctx || !ops_per_s || !ms || iters <= 0) return fail(FI8_ERR_ARG, "fi8_probe_tensor_i8: bad arguments");
  DeviceGuard g(ctx->device);
  unsigned int* d_err = nullptr;
  unsigned int h_err = 0;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaError_t e = cudaMalloc(&d_err, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemset(d_err, 0, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaEventCreate(&e0);
  if (e == cudaSuccess) e = cudaEventCreate(&e1);
  if (e == cudaSuccess) e = mma_probe_launch(ctx->sm_count, 1, d_err, nullptr);  // warm-up
  if (e == cudaSuccess) e = cudaEventRecord(e0, nullptr);
  if (e == cudaSuccess) e = mma_probe_launch(ctx->sm_count, iters, d_err, nullptr);
  if (e == cudaSuccess) e = cudaEventRecord(e1, nullptr);
  if (e == cudaSuccess) e = cudaEventSynchronize(e1);
  float dt = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&dt, e0, e1);
  if (e == cudaSuccess) e = cudaMemcpy(&h_err, d_err, sizeof(unsigned int), cudaMemcpyDeviceToHost);
  cudaFree(d_err);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (e != cudaSuccess) return cuda_fail(e, "fi8_probe_tensor_i8");
  if (h_err) return fail(FI8_ERR_DEVICE, "fi8_probe_tensor_i8: a bounded wait expired");
  *ms = dt;
  *ops_per_s = mma_probe_ops(ctx->sm_count, iters) / (dt * 1e-3);
  return FI8_OK;
}

int fi8_ctx_sm_count(fi8_ctx* ctx, int* out) {
  if (!ctx || !out) return fail(FI8_ERR_ARG, "fi8_ctx_sm_count: null argument");
  *out = ctx->sm_count;
  return FI8_OK;
}

static void index_free(fi8_index* x) {
  DeviceGuard g(x->device);
  if (x->stream) cudaStreamSynchronize(x->stream);
  delete x->up_stage;  // waits for its last copies, frees the pinned buffers
  cudaFree(x->d_codes);
  cudaFree(x->d_scales);
  cudaFree(x->d_gthr);
  cudaFree(x->d_counter);
  cudaFree(x->d_counter2);
  cudaFree(x->d_lvl1);
  cudaFree(x->d_lvl2);
  cudaFree(x->d_err);
  cudaFree(x->d_redo);
  cudaFree(x->d_q);
  cudaFree(x->d_keys);
  cudaFree(x->d_scores);
  cudaFree(x->d_A);
  cudaFree(x->d_qscale);
  cudaFree(x->d_thr);
  cudaFree(x->d_cnt);
  cudaFree(x->d_cand);
  cudaFree(x->d_topk);
  cudaFree(x->d_keep);
  if (x->h_keys) cudaFreeHost(x->h_keys);
  if (x->h_err) cudaFreeHost(x->h_err);
  for (auto& t : x->timed) {
    cudaEventDestroy(t.e0);
    cudaEventDestroy(t.e1);
  }
  for (cudaEvent_t e : x->event_pool) cudaEventDestroy(e);
  if (x->stream) cudaStreamDestroy(x->stream);
  delete x;
}

}  // extern "C"

// An index with zeroed device rows of the given shape (no data yet).
static int index_alloc(fi8_ctx* ctx, int64_t n, int32_t dim, int64_t id_base, const char* who, fi8_index** out) {
  *out = nullptr;
  if (!ctx) return fail(FI8_ERR_ARG, "%s: null ctx", who);
  if (n <= 0 || dim <= 0)  // gpu/anncuda/backend.go:125-127
    return fail(FI8_ERR_ARG, "gpu: empty int8 index (n=%lld dim=%d)", (long long)n, dim);
  if (id_base < 0 || id_base + n > 0x7FFFFFFFll)
    return fail(FI8_ERR_ARG, "%s: global indices must fit in 31 bits (id_base=%lld n=%lld)", who,
                (long long)id_base, (long long)n);
  const int32_t dpad = (dim + 15) / 16 * 16;
  if (dpad > kScanMaxDpad) return fail(FI8_ERR_DECLINED, "%s: dim %d exceeds the supported %d", who, dim, kScanMaxDpad);
  DeviceGuard g(ctx->device);
  fi8_index* x = new (std::nothrow) fi8_index;
  if (!x) return fail(FI8_ERR_OOM, "%s: host allocation", who);
  x->ctx = ctx;
  x->device = ctx->device;
  x->sm_count = ctx->sm_count;
  x->n = n;
  x->n_alloc = (n + kRowAlign - 1) / kRowAlign * kRowAlign;
  x->dim = dim;
  x->dpad = dpad;
  x->id_base = (uint32_t)id_base;
  cudaError_t e = cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&x->d_codes, (size_t)x->n_alloc * dpad);
  if (e == cudaSuccess) e = cudaMalloc(&x->d_scales, (size_t)x->n_alloc * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&x->d_err, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMalloc(&x->d_redo, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMallocHost(&x->h_err, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemsetAsync(x->d_codes, 0, (size_t)x->n_alloc * dpad, x->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(x->d_scales, 0, (size_t)x->n_alloc * sizeof(float), x->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(x->d_err, 0, sizeof(unsigned int), x->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(x->d_redo, 0, sizeof(unsigned int), x->stream);
  if (e != cudaSuccess) {
    const int rc = cuda_fail(e, "gpu: device allocation failed");
    index_free(x);
    return rc;
  }
  *out = x;
  return FI8_OK;
}

// Finish an index whose rows are on the device: wait for the uploads, build
// the corpus tensor map.
static int index_finish(fi8_index* x) {
  DeviceGuard g(x->device);
  FI8_CUDA(cudaStreamSynchronize(x->stream), "gpu: device upload failed");
  x->has_tmB = make_tmap_i8(&x->tmB, x->d_codes, (uint64_t)x->n_alloc, (uint64_t)x->dpad, (uint32_t)kGemmBN);
  x->has_tmB2 = make_tmap_i8(&x->tmB2, x->d_codes, (uint64_t)x->n_alloc, (uint64_t)x->dpad, (uint32_t)(kGemmBN / 2));
  return FI8_OK;
}

// Rows of float vectors per chunk of the device builds: one pinned buffer.
static int64_t build_chunk_rows(int32_t dim) {
  return std::max<int64_t>(1, (int64_t)(PinnedStager::kBufBytes / ((size_t)dim * 4)));
}

extern "C" {

int fi8_index_create(fi8_ctx* ctx, const int8_t* codes, const float* scales, int64_t n, int32_t dim,
                     int64_t id_base, fi8_index** out) {
  if (!out) return fail(FI8_ERR_ARG, "fi8_index_create: null out");
  *out = nullptr;
  if (n > 0 && dim > 0 && (!codes || !scales)) return fail(FI8_ERR_ARG, "fi8_index_create: null codes/scales");
  fi8_index* x = nullptr;
  int rc = index_alloc(ctx, n, dim, id_base, "fi8_index_create", &x);
  if (rc != FI8_OK) return rc;
  DeviceGuard g(x->device);
  PinnedStager stage;
  cudaError_t e = stage.init();
  if (e == cudaSuccess) e = stage.put_rows(x->d_codes, x->dpad, codes, dim, dim, n, x->stream);
  if (e == cudaSuccess) e = stage.put_rows(x->d_scales, 4, scales, 4, 4, n, x->stream);
  if (e == cudaSuccess) e = stage.finish();
  if (e != cudaSuccess || (rc = index_finish(x)) != FI8_OK) {
    if (e != cudaSuccess) rc = cuda_fail(e, "gpu: device upload failed");
    index_free(x);
    return rc;
  }
  *out = x;
  return FI8_OK;
}

int fi8_index_create_f32(fi8_ctx* ctx, const float* vecs, int64_t n, int32_t dim, int64_t id_base,
                         fi8_index** out) {
  if (!out) return fail(FI8_ERR_ARG, "fi8_index_create_f32: null out");
  *out = nullptr;
  if (n > 0 && dim > 0 && !vecs) return fail(FI8_ERR_ARG, "fi8_index_create_f32: null vectors");
  fi8_index* x = nullptr;
  int rc = index_alloc(ctx, n, dim, id_base, "fi8_index_create_f32", &x);
  if (rc != FI8_OK) return rc;
  DeviceGuard g(x->device);
  const int64_t chunk = std::min<int64_t>(n, build_chunk_rows(dim));
  float* d_v = nullptr;
  PinnedStager stage;
  cudaError_t e = stage.init();
  if (e == cudaSuccess) e = cudaMalloc(&d_v, (size_t)chunk * dim * sizeof(float));
  const size_t rb = (size_t)dim * sizeof(float);
  for (int64_t r0 = 0; e == cudaSuccess && r0 < n; r0 += chunk) {
    const int64_t rows = std::min(chunk, n - r0);
    // stream order keeps the next chunk's copy behind this chunk's kernel
    e = stage.put_rows(d_v, rb, vecs + (size_t)r0 * dim, rb, rb, rows, x->stream);
    if (e == cudaSuccess)
      e = quantize_rows_launch(d_v, rows, dim, x->dpad, x->d_codes + (size_t)r0 * x->dpad, x->d_scales + r0,
                               x->stream);
  }
  if (e == cudaSuccess) e = stage.finish();
  if (e == cudaSuccess) e = cudaStreamSynchronize(x->stream);
  cudaFree(d_v);
  if (e != cudaSuccess || (rc = index_finish(x)) != FI8_OK) {
    if (e != cudaSuccess) rc = cuda_fail(e, "gpu: device build failed");
    index_free(x);
    return rc;
  }
  *out = x;
  return FI8_OK;
}

int fi8_index_create_empty(fi8_ctx* ctx, int64_t n, int32_t dim, int64_t id_base, fi8_index** out) {
  if (!out) return fail(FI8_ERR_ARG, "fi8_index_create_empty: null out");
  *out = nullptr;
  fi8_index* x = nullptr;
  int rc = index_alloc(ctx, n, dim, id_base, "fi8_index_create_empty", &x);
  if (rc != FI8_OK) return rc;
  if ((rc = index_finish(x)) != FI8_OK) {
    index_free(x);
    return rc;
  }
  *out = x;
  return FI8_OK;
}

int fi8_index_upload_rows(fi8_index* idx, int64_t row0, const int8_t* codes, const float* scales, int64_t rows) {
  if (!idx) return fail(FI8_ERR_ARG, "fi8_index_upload_rows: null index");
  if (rows == 0) return FI8_OK;
  if (rows < 0 || row0 < 0 || row0 + rows > idx->n || !codes || !scales)
    return fail(FI8_ERR_ARG, "fi8_index_upload_rows: rows [%lld, %lld) outside [0, %lld) or null data",
                (long long)row0, (long long)(row0 + rows), (long long)idx->n);
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  if (!idx->up_stage) {
    idx->up_stage = new (std::nothrow) PinnedStager;
    if (!idx->up_stage) return fail(FI8_ERR_OOM, "fi8_index_upload_rows: host allocation");
    cudaError_t e = idx->up_stage->init();
    if (e != cudaSuccess) {
      delete idx->up_stage;
      idx->up_stage = nullptr;
      return cuda_fail(e, "gpu: pinned staging buffers");
    }
  }
  // put_rows has read the host rows when it returns (they are copied into
  // the pinned buffers); the DMA from those buffers drains on the stream
  cudaError_t e = idx->up_stage->put_rows(idx->d_codes + (size_t)row0 * idx->dpad, idx->dpad, codes, idx->dim,
                                          idx->dim, rows, idx->stream);
  if (e == cudaSuccess)
    e = idx->up_stage->put_rows(idx->d_scales + row0, 4, scales, 4, 4, rows, idx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "gpu: device upload failed");
  return FI8_OK;
}

int fi8_index_upload_finish(fi8_index* idx) {
  if (!idx) return fail(FI8_ERR_ARG, "fi8_index_upload_finish: null index");
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  if (idx->up_stage) {
    cudaError_t e = idx->up_stage->finish();
    delete idx->up_stage;
    idx->up_stage = nullptr;
    if (e != cudaSuccess) return cuda_fail(e, "gpu: device upload failed");
  }
  FI8_CUDA(cudaStreamSynchronize(idx->stream), "gpu: device upload failed");
  return FI8_OK;
}

int fi8_index_read_rows(fi8_index* idx, int8_t* codes, float* scales) {
  if (!idx || !codes || !scales) return fail(FI8_ERR_ARG, "fi8_index_read_rows: null argument");
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  fi8_index* x = idx;
  cudaError_t e;
  if (x->dpad == x->dim)
    e = cudaMemcpyAsync(codes, x->d_codes, (size_t)x->n * x->dim, cudaMemcpyDeviceToHost, x->stream);
  else
    e = cudaMemcpy2DAsync(codes, x->dim, x->d_codes, x->dpad, x->dim, (size_t)x->n, cudaMemcpyDeviceToHost,
                          x->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(scales, x->d_scales, (size_t)x->n * sizeof(float), cudaMemcpyDeviceToHost, x->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(x->stream);
  if (e != cudaSuccess) return cuda_fail(e, "fi8_index_read_rows");
  return FI8_OK;
}

int fi8_index_destroy(fi8_index* idx) {
  if (!idx) return FI8_OK;
  {
    std::lock_guard<std::mutex> lk(idx->mu);
  }
  index_free(idx);
  return FI8_OK;
}

int fi8_index_info(fi8_index* idx, int64_t* n, int32_t* dim) {
  if (!idx) return fail(FI8_ERR_ARG, "fi8_index_info: null index");
  if (n) *n = idx->n;
  if (dim) *dim = idx->dim;
  return FI8_OK;
}

int fi8_topk_max_k(fi8_index* idx, int32_t* out) {
  if (!idx || !out) return fail(FI8_ERR_ARG, "fi8_topk_max_k: null argument");
  ScanGeometry g;
  int32_t lo = 1, hi = kScanMaxCap;
  while (lo < hi) {  // largest k with a valid geometry
    const int32_t mid = (lo + hi + 1) / 2;
    if (scan_geometry(idx->dpad, mid, true, &g)) lo = mid;
    else hi = mid - 1;
  }
  *out = std::min<int32_t>(lo, kMergeMaxK);
  return FI8_OK;
}

// ---------------------------------------------------------------------------
// internal launch helpers (caller holds idx->mu and the device)
// ---------------------------------------------------------------------------

static int ensure_topk_scratch(fi8_index* x, int32_t M, int32_t kp, int32_t G, cudaStream_t st) {
  int rc;
  const int32_t NB = scan_blocks(G);
  const size_t old_gthr = x->gthr_cap, old_ctr = x->counter_cap, old_ctr2 = x->counter2_cap;
  if ((rc = ensure_device(&x->d_gthr, &x->gthr_cap, (size_t)M, "scratch gthr")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_counter, &x->counter_cap, (size_t)M * NB, "scratch counter")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_counter2, &x->counter2_cap, (size_t)M, "scratch counter2")) != FI8_OK) return rc;
  if (x->gthr_cap != old_gthr || x->counter_cap != old_ctr || x->counter2_cap != old_ctr2) {
    // Fresh (or regrown) per-query state must start at zero, ordered before the
    // kernel on its stream; the kernel returns it to zero after every launch.
    FI8_CUDA(cudaMemsetAsync(x->d_gthr, 0, x->gthr_cap * sizeof(unsigned long long), st), "memset gthr");
    FI8_CUDA(cudaMemsetAsync(x->d_counter, 0, x->counter_cap * sizeof(unsigned int), st), "memset counter");
    FI8_CUDA(cudaMemsetAsync(x->d_counter2, 0, x->counter2_cap * sizeof(unsigned int), st), "memset counter2");
  }
  if ((rc = ensure_device(&x->d_lvl1, &x->lvl1_cap, (size_t)M * G * kp, "scratch lvl1")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_lvl2, &x->lvl2_cap, (size_t)M * NB * kp, "scratch lvl2")) != FI8_OK) return rc;
  return FI8_OK;
}

static ScanParams base_params(fi8_index* x, const ScanGeometry& geo) {
  ScanParams p{};
  p.codes = x->d_codes;
  p.scales = x->d_scales;
  p.n = x->n;
  p.d = x->dim;
  p.dpad = x->dpad;
  p.rows_per_tile = geo.rows_per_tile;
  p.stages = geo.stages;
  p.ntiles = x->n_alloc / geo.rows_per_tile;
  p.id_base = x->id_base;
  p.smem_bytes = (int32_t)geo.smem_bytes;
  p.err = x->d_err;
  p.keep = x->cur_keep;
  p.keep_nbits = x->cur_keep_nbits;
  return p;
}

// Algorithmic bytes of a scan launch over mm queries: one pass over every
// row's codes and scale per query, plus the float queries.
static double scan_bytes(const fi8_index* x, int32_t mm) {
  return (double)mm * ((double)x->n * (x->dim + 4) + (double)x->dim * 4);
}

static int32_t grid_ctas(fi8_index* x, const ScanParams& p) {
  int64_t G = std::min<int64_t>(x->sm_count > 0 ? x->sm_count : 1, p.ntiles);
  return (int32_t)std::max<int64_t>(G, 1);
}

// gate: null for a plain launch; otherwise the launches are the batched
// path's exact redo and run only when *gate is set (timed as FI8_KERNEL_REDO).
static int launch_topk_scan(fi8_index* x, const float* d_q, int32_t M, int32_t k, uint64_t* d_keys,
                            cudaStream_t st, const unsigned int* gate = nullptr) {
  ScanGeometry geo;
  if (!scan_geometry(x->dpad, k, true, &geo))
    return fail(FI8_ERR_DECLINED, "gpu: TopKBatch declined (k=%d beyond the device top-K)", k);
  ScanParams p = base_params(x, geo);
  int32_t G = grid_ctas(x, p);
  int32_t Mc = std::min(M, kScanMaxM);
  if (gate) {
    // A closed gated launch costs its start plus a quick exit of each CTA, so
    // the redo takes as many queries per launch as about 32 MB of per-query
    // scratch allows (at least a wave's worth): one CTA per query, or
    // sm_count / queries CTAs each when there are fewer queries than SMs.
    // When open it streams the corpus once per query all the same. (One-wave
    // launches cost a batch of 4096 queries 29 launches and 0.21 ms.)
    const int64_t per_query = 2 * (int64_t)geo.kp * (int64_t)sizeof(uint64_t);  // lvl1 + lvl2 at G = 1
    const int64_t fit = std::min<int64_t>(65535, std::max<int64_t>(x->sm_count, (32ll << 20) / per_query));
    Mc = (int32_t)std::min<int64_t>(M, std::max<int64_t>(kScanMaxM, fit));
    G = std::max<int32_t>(1, std::min<int32_t>(G, x->sm_count / Mc));
  }
  int rc = ensure_topk_scratch(x, Mc, geo.kp, G, st);
  if (rc != FI8_OK) return rc;
  p.k = k;
  p.kp = geo.kp;
  p.cap = geo.cap;
  p.gthr = x->d_gthr;
  p.counter = x->d_counter;
  p.counter2 = x->d_counter2;
  p.lvl1 = x->d_lvl1;
  p.lvl2 = x->d_lvl2;
  p.gate = gate;
  for (int32_t m0 = 0; m0 < M; m0 += Mc) {
    const int32_t mm = std::min(Mc, M - m0);
    p.q = d_q + (size_t)m0 * x->dim;
    p.out_keys = d_keys + (size_t)m0 * k;
    cudaEvent_t t0 = timer_begin(x, st);
    cudaError_t e = scan_launch(p, true, mm, G, st);
    if (e != cudaSuccess) return cuda_fail(e, "scan_launch(topk)");
    if (gate)
      timer_end(x, st, t0, FI8_KERNEL_REDO, 0.0);
    else
      timer_end(x, st, t0, FI8_KERNEL_SCAN, scan_bytes(x, mm));
    x->last_launches++;
  }
  return FI8_OK;
}

// ---------------------------------------------------------------------------
// Batched path: quantize the batch, then for each row range one tcgen05 GEMM
// (threshold-filter epilogue) and one per-query select.
// ---------------------------------------------------------------------------
static int32_t pow2_ge_host(int64_t x) {
  int32_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Per-query candidate capacity of a batch of M: ~256 MB of keys at most
// across the batch, 8K to 64K keys per query.
static int32_t gemm_cap(int32_t M) {
  const int32_t cap = pow2_ge_host(std::max<int64_t>(8192, std::min<int64_t>(65536, (1ll << 25) / M)));
  return std::min<int32_t>(cap, 65536);
}

// CTAs of a batched GEMM launch (at most `ctas`). A CTA (or CTA pair) walks
// units strided by the grid size, so unless the grid is a multiple of the
// query tiles its query tile changes on every unit, and each change costs the
// epilogue a flush of its staged candidates and a fresh set-up of the lanes'
// per-query scale and threshold (about 90 instructions per warp). Where the
// epilogue is the GEMM's bottleneck -- rows of at most 256 bytes, whose MMA is
// short next to the epilogue of a 128 x 256 unit -- that is up to 17 % of a
// unit, so the grid drops to the largest multiple of the query tiles when that
// leaves at least 90 % of the CTAs (144 of 148 SMs at 8 query tiles). Longer
// rows hide the set-up behind the MMA and keep every SM.
static int32_t gemm_grid_ctas(int32_t ctas, int32_t wtiles, bool pair, int32_t kchunks) {
  if (kchunks > 2 || wtiles <= 0) return ctas;
  const int32_t walkers = pair ? ctas / 2 : ctas;
  const int32_t fixed = walkers / wtiles * wtiles;
  if (fixed == 0 || fixed == walkers || 10 * (int64_t)fixed < 9 * (int64_t)walkers) return ctas;
  return pair ? 2 * fixed : fixed;
}

// Row ranges [0,s1), [s1, s1*F), ... rounded to 256-row tiles. A range after
// the first admits about k*F candidates per query; every range costs a GEMM
// launch and a select.
// The first range takes every row as a candidate: max(k, 4096) rows. Its
// select is the most expensive one (a 4096-key union per query); a 16K-row
// first range cost a row shard of 1.25M rows (C2 over 8 GPUs) 10 % more per
// batch on B200, and 10M rows no less. Then two regimes:
//  * batches of up to 64 queries stream the corpus at the HBM rate and the
//    epilogue hides under the loads, so ranges are few: the growth factor is
//    64 (16 while ranges are short);
//  * larger batches are bound by the tensor pipe and the epilogue, where
//    every candidate costs epilogue and select work, so ranges are finer: the
//    growth factor is 8 (2 when k >= 512). A range growing by F admits about
//    k (F - 1) / ln F candidates per query per e-fold of rows, so at large k
//    the finer growth saves more epilogue and select work than its extra
//    launches cost. On B200 growth 4 (from 8) took a batch of 512 at k = 1000
//    from 2.73 to 2.37 ms (4M rows) and a batch of 1024 at k = 1000 from 4.04
//    to 3.67 ms, with batch 4096 at k = 100 unchanged; growth 2 then took the
//    batch of 1024 at k = 1000 over 100M rows of d = 256 from 33.7-34.0 to
//    32.0-32.4 ms and left the batch of 512 over 25M sign rows even.
// All factors stay within a quarter of the per-query buffer.
static void plan_ranges(int64_t n, int32_t M, int32_t k, int32_t cap, std::vector<GemmLevel>* out) {
  const int64_t room = std::max<int64_t>(4, cap / (4 * (int64_t)k));
  const bool fine = M > 64;
  const int64_t F1 = std::min<int64_t>(fine ? (k >= 512 ? 2 : 8) : 16, room);
  const int64_t F2 = fine ? F1 : std::min<int64_t>(64, room);
  int64_t hi = std::max<int64_t>(k, 4096);
  hi = (hi + kGemmBN - 1) / kGemmBN * kGemmBN;
  int64_t lo = 0;
  while (lo < n) {
    int64_t h = std::min<int64_t>(n, hi);
    // a short tail after this range joins it when the joined range still
    // admits few enough candidates (about k * (h - lo) / lo per query): one
    // launch and one select fewer, which matters on small row shards
    if (lo > 0 && h < n && n - h < (h - lo) / 2 && n - lo <= lo * room) h = n;
    out->push_back(GemmLevel{lo, h});
    lo = h;
    const int64_t F = lo >= 16 * 1024 ? F2 : F1;
    hi = (lo * F + kGemmBN - 1) / kGemmBN * kGemmBN;
  }
}

// The corpus side of a batched top-k GEMM: FlatI8's int8 rows scored W8A8, or
// a binary index's sign rows (+1/-1 per code bit) scored by -Hamming distance.
struct GemmCorpus {
  const CUtensorMap* tmB;  // [n_alloc][dpad] int8 rows, 256-row boxes
  const CUtensorMap* tmB2; // the same rows in 128-row boxes (null: no CTA pairs)
  const float* scales;     // W8A8: the row scales; null in Hamming mode
  const float* center;     // Hamming mode: the prefilter's centre (null: none)
  int32_t ham_dim;         // > 0: Hamming mode over this many bits
};

static int launch_topk_gemm(fi8_index* x, const GemmCorpus& corpus, const float* d_q, int32_t M, int32_t k,
                            uint64_t* d_keys, cudaStream_t st) {
  if (k > select_max_k())
    return fail(FI8_ERR_DECLINED, "gpu: TopKBatch declined (k=%d beyond the device top-K)", k);
  const int32_t kp = pow2_ge_host(k);
  const int32_t bm = M <= 64 ? 64 : kGemmBM;  // the MMA's M: a small batch is one 64-query tile
  // Batches of more than one 128-query tile are tensor-bound: they run on CTA
  // pairs (256-query x 256-row units, 2/3 of the operand bytes per SM).
  const int32_t pair_clusters = gemm_pair_max_clusters();
  const bool pair = x->gemm_pair && M > kGemmBM && corpus.tmB2 && pair_clusters > 0;
  const int32_t Mpad = pair ? (M + 2 * kGemmBM - 1) / (2 * kGemmBM) * (2 * kGemmBM) : (M + bm - 1) / bm * bm;
  const int32_t cap = gemm_cap(M);
  int rc;
  if ((rc = ensure_device(&x->d_A, &x->A_cap, (size_t)Mpad * x->dpad, "gemm A")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_qscale, &x->qscale_cap, (size_t)Mpad, "gemm qscale")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_thr, &x->thr_cap, (size_t)M, "gemm thr")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_cnt, &x->cnt_cap, (size_t)M, "gemm cnt")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_cand, &x->cand_cap, (size_t)M * cap, "gemm cand")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_topk, &x->topk_cap, (size_t)M * kp, "gemm topk")) != FI8_OK) return rc;
  const int64_t A_rows = (int64_t)(x->A_cap / x->dpad);
  if (x->tmA_base != x->d_A || x->tmA_rows != A_rows || x->tmA_box != bm) {
    if (!make_tmap_i8(&x->tmA, x->d_A, (uint64_t)A_rows, (uint64_t)x->dpad, (uint32_t)bm))
      return fail(FI8_ERR_CUDA, "fi8: cuTensorMapEncodeTiled failed for the query tile map");
    x->tmA_base = x->d_A;
    x->tmA_rows = A_rows;
    x->tmA_box = bm;
  }
  cudaEvent_t t0 = timer_begin(x, st);
  const bool ham = corpus.ham_dim > 0;
  cudaError_t e = ham ? sign_prep_launch(d_q, M, Mpad, x->dim, x->dpad, corpus.center, x->d_A, x->d_qscale,
                                         x->d_thr, x->d_cnt, x->d_topk, kp, bm, st)
                      : quantize_launch(d_q, M, Mpad, x->dim, x->dpad, x->d_A, x->d_qscale, x->d_thr, x->d_cnt,
                                        x->d_topk, kp, bm, st);
  if (e != cudaSuccess) return cuda_fail(e, ham ? "sign_prep_launch" : "quantize_launch");
  timer_end(x, st, t0, FI8_KERNEL_QUANTIZE, (double)M * x->dim * 4 + (double)Mpad * x->dpad);
  x->last_launches++;
  std::vector<GemmLevel> ranges;
  plan_ranges(x->n, M, k, cap, &ranges);
  GemmParams p{};
  p.kchunks = (x->dpad + kGemmBK - 1) / kGemmBK;
  p.M = M;
  p.qtiles = Mpad / bm;
  p.id_base = x->id_base;
  p.scales = corpus.scales;
  p.ham_dim = corpus.ham_dim;
  p.qscale = x->d_qscale;
  p.thr = x->d_thr;
  p.cnt = x->d_cnt;
  p.cand = x->d_cand;
  p.cap = cap;
  p.err = x->d_err;
  p.keep = x->cur_keep;
  p.keep_nbits = x->cur_keep_nbits;
  for (size_t i = 0; i < ranges.size(); i++) {
    p.row_lo = ranges[i].row_lo;
    p.row_hi = ranges[i].row_hi;
    p.rtiles = (p.row_hi - p.row_lo + kGemmBN - 1) / kGemmBN;
    p.producer_waits = i == 0 ? 1 : 0;  // the first range follows the quantize kernel
    const int32_t wtiles = pair ? p.qtiles / 2 : p.qtiles;  // query tiles of the unit walk
    const int64_t units = (int64_t)wtiles * p.rtiles;
    const int32_t ctas = gemm_grid_ctas(x->gemm_ctas > 0 ? std::min(x->gemm_ctas, x->sm_count) : x->sm_count,
                                        wtiles, pair, p.kchunks);
    // CTAs: one per SM, or pairs of them, no more than there are units
    const int32_t G = pair ? 2 * (int32_t)std::max<int64_t>(1, std::min<int64_t>({(int64_t)ctas / 2,
                                                                                   (int64_t)pair_clusters, units}))
                           : (int32_t)std::max<int64_t>(1, std::min<int64_t>(ctas, units));
    t0 = timer_begin(x, st);
    e = gemm_launch(x->tmA, pair ? *corpus.tmB2 : *corpus.tmB, p, G, bm, pair, st);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_launch");
    // the range's rows (and scales), plus the int8 query tile
    timer_end(x, st, t0, FI8_KERNEL_GEMM,
              (double)(p.row_hi - p.row_lo) * (x->dim + (ham ? 0 : 4)) + (double)M * x->dim);
    const bool last = (i + 1 == ranges.size());
    t0 = timer_begin(x, st);
    e = select_launch(M, k, kp, x->d_topk, x->d_thr, x->d_cnt, x->d_cand, cap, last ? d_keys : nullptr,
                      x->d_err, x->sm_count, st);
    if (e != cudaSuccess) return cuda_fail(e, "select_launch");
    timer_end(x, st, t0, FI8_KERNEL_SELECT, 0.0);
    x->last_launches += 2;
  }
  return FI8_OK;
}

// After a batched top-k: the latch moves the selects' dropped-candidate flag
// into the index's redo gate, then the per-query scan (which has no
// candidate buffer) recomputes the batch into d_keys, gated on that flag. The
// gated launches return at once when nothing was dropped, so every answer is
// exact in stream order, with no host round trip. When no scan form exists
// for this k the flag stays set and surfaces at the next sync.
static int launch_topk_redo(fi8_index* x, const float* d_q, int32_t M, int32_t k, uint64_t* d_keys,
                            cudaStream_t st) {
  ScanGeometry geo;
  if (!scan_geometry(x->dpad, k, true, &geo)) return FI8_OK;
  cudaEvent_t t0 = timer_begin(x, st);
  cudaError_t e = overflow_latch_launch(x->d_err, x->d_redo, st);
  if (e != cudaSuccess) return cuda_fail(e, "overflow_latch_launch");
  timer_end(x, st, t0, FI8_KERNEL_REDO, 0.0);
  x->last_launches++;
  return launch_topk_scan(x, d_q, M, k, d_keys, st, x->d_redo);
}

static int launch_topk(fi8_index* x, const float* d_q, int32_t M, int32_t k, uint64_t* d_keys,
                       cudaStream_t st) {
  x->last_launches = 0;
  if (M >= x->gemm_min_batch && x->has_tmB) {
    const int rc = launch_topk_gemm(x, GemmCorpus{&x->tmB, x->has_tmB2 ? &x->tmB2 : nullptr, x->d_scales, nullptr, 0},
                                    d_q, M, k, d_keys, st);
    if (rc != FI8_OK) return rc;
    return launch_topk_redo(x, d_q, M, k, d_keys, st);
  }
  return launch_topk_scan(x, d_q, M, k, d_keys, st);
}

static int launch_scores(fi8_index* x, const float* d_q, int32_t M, float* d_scores, cudaStream_t st) {
  ScanGeometry geo;
  if (!scan_geometry(x->dpad, 0, false, &geo)) return fail(FI8_ERR_ARG, "fi8: bad row pitch %d", x->dpad);
  ScanParams p = base_params(x, geo);
  const int32_t G = grid_ctas(x, p);
  for (int32_t m0 = 0; m0 < M; m0 += kScanMaxM) {
    const int32_t mm = std::min(kScanMaxM, M - m0);
    p.q = d_q + (size_t)m0 * x->dim;
    p.out_scores = d_scores + (size_t)m0 * x->n;
    cudaEvent_t t0 = timer_begin(x, st);
    cudaError_t e = scan_launch(p, false, mm, G, st);
    if (e != cudaSuccess) return cuda_fail(e, "scan_launch(score)");
    timer_end(x, st, t0, FI8_KERNEL_SCAN, scan_bytes(x, mm) + (double)mm * x->n * 4);
    x->last_launches++;
  }
  return FI8_OK;
}

// After a synchronize: surface and clear the device error flag.
static int check_device_error(fi8_index* x) {
  if (*x->h_err != 0) {
    const unsigned v = *x->h_err;
    *x->h_err = 0;
    cudaMemsetAsync(x->d_err, 0, sizeof(unsigned int), x->stream);
    if (v & 1u) {
      // a launch gave up on a wait: return the scan's cross-CTA state to zero
      // in case it stopped before its last CTA reset it
      if (x->d_gthr) cudaMemsetAsync(x->d_gthr, 0, x->gthr_cap * sizeof(unsigned long long), x->stream);
      if (x->d_counter) cudaMemsetAsync(x->d_counter, 0, x->counter_cap * sizeof(unsigned int), x->stream);
      if (x->d_counter2) cudaMemsetAsync(x->d_counter2, 0, x->counter2_cap * sizeof(unsigned int), x->stream);
    }
    cudaStreamSynchronize(x->stream);
    return fail(FI8_ERR_DEVICE, "fi8: kernel reported device error flags 0x%x (%s)", v,
                (v & 1u) ? "a bounded wait expired" : "a candidate buffer overflowed");
  }
  return FI8_OK;
}

int fi8_score_batch(fi8_index* idx, const float* q, int32_t M, float* dst) {
  if (!idx) return fail(FI8_ERR_ARG, "fi8_score_batch: null index");
  if (M == 0) return FI8_OK;
  if (M < 0 || !q || !dst) return fail(FI8_ERR_ARG, "fi8_score_batch: bad arguments");
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  fi8_index* x = idx;
  int rc;
  if ((rc = ensure_device(&x->d_q, &x->d_q_cap, (size_t)M * x->dim, "staging q")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_scores, &x->d_scores_cap, (size_t)M * x->n, "staging scores")) != FI8_OK)
    return rc;
  x->last_launches = 0;
  FI8_CUDA(cudaMemcpyAsync(x->d_q, q, (size_t)M * x->dim * sizeof(float), cudaMemcpyHostToDevice, x->stream),
           "H2D queries");
  if ((rc = launch_scores(x, x->d_q, M, x->d_scores, x->stream)) != FI8_OK) return rc;
  FI8_CUDA(cudaMemcpyAsync(dst, x->d_scores, (size_t)M * x->n * sizeof(float), cudaMemcpyDeviceToHost, x->stream),
           "D2H scores");
  FI8_CUDA(cudaMemcpyAsync(x->h_err, x->d_err, sizeof(unsigned int), cudaMemcpyDeviceToHost, x->stream),
           "D2H err");
  FI8_CUDA(cudaStreamSynchronize(x->stream), "sync");
  return check_device_error(x);
}

int fi8_score(fi8_index* idx, const float* q, float* dst) { return fi8_score_batch(idx, q, 1, dst); }

}  // extern "C"

// The keep filter of one call: set on entry, cleared on every exit path.
struct KeepScope {
  fi8_index* x;
  KeepScope(fi8_index* ix, const uint64_t* keep, int64_t nbits) : x(ix) {
    x->cur_keep = keep;
    x->cur_keep_nbits = keep ? nbits : 0;
  }
  ~KeepScope() {
    x->cur_keep = nullptr;
    x->cur_keep_nbits = 0;
  }
};

// Copy a host keep bitmap (nbits bits over global ids) to the index's device
// buffer on its stream; returns the device pointer through *out.
static int stage_keep(fi8_index* x, const uint64_t* keep, int64_t nbits, const uint64_t** out) {
  *out = nullptr;
  if (!keep) return FI8_OK;
  if (nbits < 0) return fail(FI8_ERR_ARG, "fi8: keep bitmap with negative length");
  const size_t words = (size_t)((nbits + 63) / 64);
  int rc;
  if ((rc = ensure_device(&x->d_keep, &x->keep_cap, words, "keep bitmap")) != FI8_OK) return rc;
  if (words)
    FI8_CUDA(cudaMemcpyAsync(x->d_keep, keep, words * 8, cudaMemcpyHostToDevice, x->stream), "H2D keep");
  *out = x->d_keep;
  return FI8_OK;
}

// Top-k of the M queries staged in x->d_q into x->h_keys (M*k keys). A
// batched answer that dropped candidates is redone on the device inside
// launch_topk. Caller holds x->mu and the device.
static int topk_staged(fi8_index* x, int32_t M, int32_t k) {
  const size_t nk = (size_t)M * k;
  int rc;
  if ((rc = ensure_device(&x->d_keys, &x->d_keys_cap, nk, "staging keys")) != FI8_OK) return rc;
  if ((rc = ensure_host(&x->h_keys, &x->h_keys_cap, nk, "pinned keys")) != FI8_OK) return rc;
  if ((rc = launch_topk(x, x->d_q, M, k, x->d_keys, x->stream)) != FI8_OK) return rc;
  FI8_CUDA(cudaMemcpyAsync(x->h_keys, x->d_keys, nk * sizeof(uint64_t), cudaMemcpyDeviceToHost, x->stream),
           "D2H keys");
  FI8_CUDA(cudaMemcpyAsync(x->h_err, x->d_err, sizeof(unsigned int), cudaMemcpyDeviceToHost, x->stream),
           "D2H err");
  FI8_CUDA(cudaStreamSynchronize(x->stream), "sync");
  return check_device_error(x);
}

extern "C" {

int fi8_topk_batch_keep(fi8_index* idx, const float* q, int32_t M, int32_t k, const uint64_t* keep, int64_t nbits,
                        int32_t* out_idx, float* out_score) {
  if (!idx) return fail(FI8_ERR_ARG, "fi8_topk_batch: null index");
  if (M == 0) return FI8_OK;
  if (M < 0 || !q || !out_idx || !out_score) return fail(FI8_ERR_ARG, "fi8_topk_batch: bad arguments");
  if (k <= 0 || (int64_t)k >= idx->n)  // gpu/anncuda/backend.go:577-579
    return fail(FI8_ERR_DECLINED, "gpu: TopKBatch declined (k=%d n=%lld batch=%d)", k, (long long)idx->n, M);
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  fi8_index* x = idx;
  int rc;
  const uint64_t* d_keep = nullptr;
  if ((rc = stage_keep(x, keep, nbits, &d_keep)) != FI8_OK) return rc;
  KeepScope ks(x, d_keep, nbits);
  if ((rc = ensure_device(&x->d_q, &x->d_q_cap, (size_t)M * x->dim, "staging q")) != FI8_OK) return rc;
  FI8_CUDA(cudaMemcpyAsync(x->d_q, q, (size_t)M * x->dim * sizeof(float), cudaMemcpyHostToDevice, x->stream),
           "H2D queries");
  if ((rc = topk_staged(x, M, k)) != FI8_OK) return rc;
  return fi8_keys_unpack(x->h_keys, (int64_t)M * k, out_idx, out_score);
}

int fi8_topk_batch(fi8_index* idx, const float* q, int32_t M, int32_t k, int32_t* out_idx, float* out_score) {
  return fi8_topk_batch_keep(idx, q, M, k, nullptr, 0, out_idx, out_score);
}

int fi8_topk_batch_async_keep(fi8_index* idx, const float* d_q, int32_t M, int32_t k, const uint64_t* d_keep,
                              int64_t nbits, uint64_t* d_keys, void* stream) {
  if (!idx) return fail(FI8_ERR_ARG, "fi8_topk_batch_async: null index");
  if (M == 0) return FI8_OK;
  if (M < 0 || !d_q || !d_keys || nbits < 0) return fail(FI8_ERR_ARG, "fi8_topk_batch_async: bad arguments");
  // k >= n is allowed here: a row shard smaller than k contributes all of its
  // rows (sorted, then empty slots) to the cross-shard merge.
  if (k <= 0) return fail(FI8_ERR_DECLINED, "gpu: TopKBatch declined (k=%d)", k);
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  KeepScope ks(idx, d_keep, nbits);
  return launch_topk(idx, d_q, M, k, d_keys, static_cast<cudaStream_t>(stream));
}

int fi8_topk_batch_async(fi8_index* idx, const float* d_q, int32_t M, int32_t k, uint64_t* d_keys,
                         void* stream) {
  return fi8_topk_batch_async_keep(idx, d_q, M, k, nullptr, 0, d_keys, stream);
}

int fi8_index_set_option(fi8_index* idx, int option, int64_t value) {
  if (!idx) return fail(FI8_ERR_ARG, "fi8_index_set_option: null index");
  std::lock_guard<std::mutex> lk(idx->mu);
  switch (option) {
    case FI8_OPT_GEMM_MIN_BATCH:
      if (value < 1) return fail(FI8_ERR_ARG, "fi8_index_set_option: GEMM_MIN_BATCH must be >= 1");
      idx->gemm_min_batch = (int32_t)std::min<int64_t>(value, 1 << 30);
      return FI8_OK;
    case FI8_OPT_KERNEL_TIMING:
      if (value != 0 && value != 1) return fail(FI8_ERR_ARG, "fi8_index_set_option: KERNEL_TIMING is 0 or 1");
      idx->timing = value != 0;
      return FI8_OK;
    case FI8_OPT_GEMM_CTAS:
      if (value < 0) return fail(FI8_ERR_ARG, "fi8_index_set_option: GEMM_CTAS must be >= 0");
      idx->gemm_ctas = (int32_t)std::min<int64_t>(value, 1 << 30);
      return FI8_OK;
    case FI8_OPT_GEMM_PAIR:
      if (value != 0 && value != 1) return fail(FI8_ERR_ARG, "fi8_index_set_option: GEMM_PAIR is 0 or 1");
      idx->gemm_pair = (int32_t)value;
      return FI8_OK;
    default:
      return fail(FI8_ERR_ARG, "fi8_index_set_option: unknown option %d", option);
  }
}

int fi8_index_last_launch_count(fi8_index* idx, int32_t* out) {
  if (!idx || !out) return fail(FI8_ERR_ARG, "fi8_index_last_launch_count: null argument");
  std::lock_guard<std::mutex> lk(idx->mu);
  *out = idx->last_launches;
  return FI8_OK;
}

int fi8_index_kernel_times(fi8_index* idx, int64_t* launches, double* ms, double* bytes, int reset) {
  if (!idx || !launches || !ms || !bytes) return fail(FI8_ERR_ARG, "fi8_index_kernel_times: null argument");
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  for (int i = 0; i < FI8_KERNEL_KINDS; i++) {
    launches[i] = 0;
    ms[i] = 0.0;
    bytes[i] = 0.0;
  }
  for (const auto& t : idx->timed) {
    FI8_CUDA(cudaEventSynchronize(t.e1), "fi8_index_kernel_times: event sync");
    float dt = 0.0f;
    FI8_CUDA(cudaEventElapsedTime(&dt, t.e0, t.e1), "fi8_index_kernel_times: elapsed time");
    launches[t.kind] += 1;
    ms[t.kind] += dt;
    bytes[t.kind] += t.bytes;
  }
  if (reset) {
    for (const auto& t : idx->timed) {
      idx->event_pool.push_back(t.e0);
      idx->event_pool.push_back(t.e1);
    }
    idx->timed.clear();
  }
  return FI8_OK;
}

int fi8_index_kernel_log(fi8_index* idx, int32_t cap, int32_t* count, int32_t* kinds, double* ms, double* bytes) {
  if (!idx || !count || (cap > 0 && (!kinds || !ms || !bytes)))
    return fail(FI8_ERR_ARG, "fi8_index_kernel_log: null argument");
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  int32_t c = 0;
  for (const auto& t : idx->timed) {
    if (c >= cap) break;
    FI8_CUDA(cudaEventSynchronize(t.e1), "fi8_index_kernel_log: event sync");
    float dt = 0.0f;
    FI8_CUDA(cudaEventElapsedTime(&dt, t.e0, t.e1), "fi8_index_kernel_log: elapsed time");
    kinds[c] = t.kind;
    ms[c] = dt;
    bytes[c] = t.bytes;
    c++;
  }
  *count = c;
  return FI8_OK;
}

int fi8_index_sync(fi8_index* idx) {
  if (!idx) return fail(FI8_ERR_ARG, "fi8_index_sync: null index");
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  FI8_CUDA(cudaDeviceSynchronize(), "sync");
  FI8_CUDA(cudaMemcpy(idx->h_err, idx->d_err, sizeof(unsigned int), cudaMemcpyDeviceToHost), "D2H err");
  return check_device_error(idx);
}

int fi8_keys_unpack(const uint64_t* keys, int64_t count, int32_t* out_idx, float* out_score) {
  if (count < 0 || (count > 0 && (!keys || !out_idx || !out_score)))
    return fail(FI8_ERR_ARG, "fi8_keys_unpack: bad arguments");
  for (int64_t i = 0; i < count; i++) {
    const uint64_t key = keys[i];
    if (key == kEmptyKey) {
      out_idx[i] = -1;
      out_score[i] = 0.0f;
    } else {
      out_idx[i] = key_index(key);
      out_score[i] = key_score(key);
    }
  }
  return FI8_OK;
}

int fi8_merge_keys_async(fi8_ctx* ctx, const uint64_t* d_in, int32_t nsrc, int32_t M, int32_t k,
                         uint64_t* d_out, void* stream) {
  if (!ctx || !d_in || !d_out) return fail(FI8_ERR_ARG, "fi8_merge_keys_async: null argument");
  if (M == 0) return FI8_OK;
  if (M < 0 || nsrc <= 0 || k <= 0) return fail(FI8_ERR_ARG, "fi8_merge_keys_async: bad shape");
  if (k > kMergeMaxK) return fail(FI8_ERR_DECLINED, "fi8_merge_keys_async: k=%d beyond %d", k, kMergeMaxK);
  DeviceGuard g(ctx->device);
  cudaError_t e = merge_keys_launch(d_in, nsrc, M, k, d_out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "merge_keys_launch");
  return FI8_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free single-query top-K (fi8_topk1_noalloc).
//
// For callers that must not allocate device memory while serving: a process
// whose HBM is pre-reserved at start-up (the corpus plus a caching allocator's
// pool) can see cudaMalloc fail on the query path, and cudaMalloc may
// synchronize the device, stalling every other stream. fi8_topk_batch_async
// grows its scratch with cudaMalloc on first use; this variant runs the same
// scan kernel with its scratch in the fixed array below instead, and calls no
// cudaMalloc, cudaFree or allocating library routine.
//
// The array exists once per device that loads this library and lives until
// the process exits. It holds, for one query: the shared threshold and the
// ticket counters (cleared before every call), kNoAllocMaxCtas per-CTA lists
// and their per-block lists of up to kNoAllocMaxK keys. Every call on a device
// shares it and it keeps the last call's contents, so two calls that overlap
// on the GPU (on different streams, or on different indexes of the same
// device) race; serialize them, e.g. on one stream.
// ---------------------------------------------------------------------------
namespace {
constexpr int32_t kNoAllocMaxK = 256;      // keys per list (k rounded up to a power of two)
constexpr int32_t kNoAllocMaxCtas = 160;   // >= the 148 SMs of a B200
constexpr int32_t kNoAllocMaxBlocks = (kNoAllocMaxCtas + kMergeBlock - 1) / kMergeBlock;
constexpr size_t kNoAllocHeader = 256;     // gthr @0, counter2 @8, counter[] @16
constexpr size_t kNoAllocLvl1 = (size_t)kNoAllocMaxCtas * kNoAllocMaxK * sizeof(uint64_t);
constexpr size_t kNoAllocLvl2 = (size_t)kNoAllocMaxBlocks * kNoAllocMaxK * sizeof(uint64_t);
constexpr size_t kNoAllocBytes = kNoAllocHeader + kNoAllocLvl1 + kNoAllocLvl2;  // 368,896 bytes
static_assert(16 + kNoAllocMaxBlocks * sizeof(unsigned int) <= kNoAllocHeader, "header overflow");

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[64] = {};  // device address of the array, per device ordinal
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

extern "C" int fi8_topk1_noalloc(fi8_index* idx, const float* d_q, int32_t k, uint64_t* d_keys, void* stream) {
  if (!idx || !d_q || !d_keys) return fail(FI8_ERR_ARG, "fi8_topk1_noalloc: null argument");
  if (k <= 0) return fail(FI8_ERR_DECLINED, "gpu: TopKBatch declined (k=%d)", k);
  if (k > kNoAllocMaxK)
    return fail(FI8_ERR_ARG, "fi8_topk1_noalloc: k=%d exceeds the allocation-free limit of %d", k, kNoAllocMaxK);
  ScanGeometry geo;
  if (!scan_geometry(idx->dpad, k, true, &geo) || geo.kp > kNoAllocMaxK)
    return fail(FI8_ERR_ARG, "fi8_topk1_noalloc: k=%d not supported for dim %d", k, idx->dim);
  std::lock_guard<std::mutex> lk(idx->mu);
  DeviceGuard g(idx->device);
  if (idx->device < 0 || idx->device >= 64) return fail(FI8_ERR_ARG, "fi8_topk1_noalloc: device ordinal");
  unsigned char* base;
  {
    // Set-up, once per device and with that device current: in host code the
    // array's name is only a stand-in, so ask the runtime for its address.
    std::lock_guard<std::mutex> lk2(g_noalloc_mu);
    if (!g_noalloc_ptr[idx->device]) {
      void* ptr = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "fi8_topk1_noalloc: cudaGetSymbolAddress");
      g_noalloc_ptr[idx->device] = static_cast<unsigned char*>(ptr);
    }
    base = g_noalloc_ptr[idx->device];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  FI8_CUDA(cudaMemsetAsync(base, 0, kNoAllocHeader, st), "fi8_topk1_noalloc: clear counters");
  ScanParams p = base_params(idx, geo);
  const int32_t G = std::min<int32_t>(grid_ctas(idx, p), kNoAllocMaxCtas);
  p.k = k;
  p.kp = geo.kp;
  p.cap = geo.cap;
  p.gthr = reinterpret_cast<unsigned long long*>(base);
  p.counter2 = reinterpret_cast<unsigned int*>(base + 8);
  p.counter = reinterpret_cast<unsigned int*>(base + 16);
  p.lvl1 = reinterpret_cast<uint64_t*>(base + kNoAllocHeader);
  p.lvl2 = reinterpret_cast<uint64_t*>(base + kNoAllocHeader + kNoAllocLvl1);
  p.q = d_q;
  p.out_keys = d_keys;
  cudaError_t e = scan_launch(p, true, 1, G, st);
  if (e != cudaSuccess) return cuda_fail(e, "fi8_topk1_noalloc: scan_launch");
  idx->last_launches = 1;
  return FI8_OK;
}

// ---------------------------------------------------------------------------
// FlatBinaryI8 (ann/flat_binary_i8.go): a device-resident sign-bit prefilter
// over an int8 FlatI8 shard. The reference has no device seam for it; this is
// additive surface for an optional BinaryI8Index-style interface.
// ---------------------------------------------------------------------------
struct fi8_bin {
  fi8_index* ix = nullptr;      // the int8 rows: rerank and the exact fallback
  int32_t words = 0;            // ceil(dim / 64) (linalg.PackedWords)
  int32_t wpad = 0;             // row pitch in words (words rounded up to even)
  int32_t over = 1;             // overquery (max(overquery, 1), prefilter.go:58)
  uint64_t* d_bits = nullptr;   // [n_alloc][wpad] packed sign bits, zero padded
  float* d_center = nullptr;    // [dim], or null for an uncentred prefilter
  // per-call scratch, grown on demand
  uint64_t* d_qbits = nullptr;  // [M][wpad] packed query bits
  size_t qbits_cap = 0;
  uint16_t* d_dist = nullptr;   // [M][n_alloc] Hamming distances
  size_t dist_cap = 0;
  unsigned int* d_hist = nullptr;    // [M][nbins]
  size_t hist_cap = 0;
  unsigned int* d_counts = nullptr;  // [M][P][2]
  size_t counts_cap = 0;
  uint64_t* d_parts = nullptr;  // [parts][M][k] rerank slices
  size_t parts_cap = 0;
  uint64_t* d_short = nullptr;  // [M][cand] shortlist keys (host entry point)
  size_t short_cap = 0;
  // tensor-core prefilter (fi8_bin_set_tensor_prefilter): the codes unpacked
  // to +1/-1 int8 rows, so a batch's Hamming distances are one kind::i8 GEMM
  int8_t* d_sign = nullptr;     // [n_alloc][dpad]; 0 past dim and for rows >= n
  CUtensorMap tmS;              // over d_sign, 256-row boxes
  CUtensorMap tmS2;             // over d_sign, 128-row boxes (CTA pairs)
  bool has_tmS2 = false;
  int32_t tensor_min_m = 0;     // batches of at least this many queries use it (0: off)
};

namespace {
// Shortlists the key merge (cross-shard), the shortlist sort and the rerank
// support.
constexpr int32_t kBinMaxCand = kMergeMaxK < kRerankMaxCand ? kMergeMaxK : kRerankMaxCand;
// Queries per distance pass: bounds the distance scratch (M x n u16).
constexpr int32_t kBinMaxM = 16;
}  // namespace

// The popcount prefilter (packing, the distance pass with its histogram, the
// cut and the shortlist) for M queries. sorted: each query's keys sorted
// descending, as a cross-shard key merge needs. gate: null for a plain
// launch; otherwise the launches are the exact redo of a tensor-core
// shortlist and run only when *gate is set (timed as FI8_KERNEL_REDO).
// Caller holds b->ix->mu and the device.
static int launch_bin_popcount(fi8_bin* b, const float* d_q, int32_t M, int32_t cand, uint64_t* d_keys,
                               bool sorted, cudaStream_t st, const unsigned int* gate = nullptr) {
  fi8_index* x = b->ix;
  const int32_t bpad = b->wpad * 8;
  const int32_t nbins = bpad * 8 + 1;
  ScanGeometry geo;
  if (cand > kBinMaxCand || !scan_geometry(bpad, 0, false, &geo, true))
    return fail(FI8_ERR_DECLINED, "gpu: binary prefilter declined (cand=%d beyond %d)", cand, kBinMaxCand);
  int32_t Mc = std::min(M, kBinMaxM);
  int32_t P = shortlist_segments(x->sm_count);
  if (gate) {
    // The gated redo's launches cost their CTAs' start and exit even when
    // closed, so each keeps to about one wave: up to 64 queries per pass
    // (16 when their distance rows would pass 4 GB), sm_count / queries CTAs
    // and row segments each. When open, every SM still streams the codes.
    Mc = std::min<int32_t>(M, (size_t)64 * x->n_alloc * sizeof(uint16_t) <= ((size_t)4 << 30) ? 64 : kBinMaxM);
    P = std::max<int32_t>(1, x->sm_count / Mc);
  }
  int rc;
  if ((rc = ensure_device(&b->d_qbits, &b->qbits_cap, (size_t)Mc * b->wpad, "binary query bits")) != FI8_OK)
    return rc;
  if ((rc = ensure_device(&b->d_dist, &b->dist_cap, (size_t)Mc * x->n_alloc, "binary distances")) != FI8_OK)
    return rc;
  if ((rc = ensure_device(&b->d_hist, &b->hist_cap, (size_t)Mc * nbins, "binary histogram")) != FI8_OK) return rc;
  if ((rc = ensure_device(&b->d_counts, &b->counts_cap, (size_t)Mc * P * 2, "binary counts")) != FI8_OK) return rc;
  ScanParams p = base_params(x, geo);
  p.codes = reinterpret_cast<const int8_t*>(b->d_bits);
  p.scales = nullptr;
  p.dpad = bpad;
  p.out_dist = b->d_dist;
  p.dist_stride = x->n_alloc;
  p.hist = b->d_hist;
  p.nbins = nbins;
  p.qbits = b->d_qbits;
  p.gate = gate;
  int32_t G = grid_ctas(x, p);
  if (gate) G = std::max<int32_t>(1, std::min<int32_t>(G, x->sm_count / Mc));
  auto timed = [&](cudaEvent_t t0, int kind, double bytes) {
    if (gate)
      timer_end(x, st, t0, FI8_KERNEL_REDO, 0.0);
    else
      timer_end(x, st, t0, kind, bytes);
  };
  for (int32_t m0 = 0; m0 < M; m0 += Mc) {
    const int32_t mm = std::min(Mc, M - m0);
    const float* q = d_q + (size_t)m0 * x->dim;
    cudaEvent_t t0 = timer_begin(x, st);
    cudaError_t e = binary_prep_launch(q, mm, x->dim, b->d_center, b->wpad, b->d_qbits, b->d_hist, nbins, st, gate);
    if (e != cudaSuccess) return cuda_fail(e, "binary_prep_launch");
    timed(t0, FI8_KERNEL_QUANTIZE, (double)mm * x->dim * 4);
    t0 = timer_begin(x, st);
    e = scan_launch(p, false, mm, G, st, true);
    if (e != cudaSuccess) return cuda_fail(e, "scan_launch(binary)");
    // the packed codes once per query, plus the u16 distance written per row
    timed(t0, FI8_KERNEL_SCAN, (double)mm * ((double)x->n * bpad + (double)bpad + 2.0 * x->n));
    t0 = timer_begin(x, st);
    e = shortlist_launch(b->d_dist, x->n, x->n_alloc, mm, b->d_hist, nbins, cand, P, b->d_counts, x->id_base,
                         d_keys + (size_t)m0 * cand, sorted, st, gate);
    if (e != cudaSuccess) return cuda_fail(e, "shortlist_launch");
    timed(t0, FI8_KERNEL_SELECT, (double)mm * 2.0 * 2.0 * x->n);
    x->last_launches += sorted ? 5 : 4;
  }
  return FI8_OK;
}

// The prefilter for M queries: the tensor-core GEMM for batches of at least
// the tensor-prefilter size (with its gated popcount redo after it: a row
// range that admitted more candidates than its per-query buffer holds, e.g.
// on a corpus ordered against the query, leaves an incomplete shortlist,
// which the popcount pass, without such a buffer, recomputes exactly), the
// popcount pass otherwise. Caller holds b->ix->mu and the device.
static int launch_bin_prefilter(fi8_bin* b, const float* d_q, int32_t M, int32_t cand, uint64_t* d_keys,
                                bool sorted, cudaStream_t st) {
  fi8_index* x = b->ix;
  if (b->d_sign && b->tensor_min_m > 0 && M >= b->tensor_min_m) {
    // The shortlist is the cand best rows under (distance asc, id asc); as
    // packed keys (-distance, id) that is the exact top-cand the GEMM path
    // selects, sorted descending (so it also serves a key merge).
    if (cand > kBinMaxCand)
      return fail(FI8_ERR_DECLINED, "gpu: binary prefilter declined (cand=%d beyond %d)", cand, kBinMaxCand);
    int rc = launch_topk_gemm(x, GemmCorpus{&b->tmS, b->has_tmS2 ? &b->tmS2 : nullptr, nullptr, b->d_center, x->dim},
                              d_q, M, cand, d_keys, st);
    if (rc != FI8_OK) return rc;
    cudaEvent_t t0 = timer_begin(x, st);
    cudaError_t e = overflow_latch_launch(x->d_err, x->d_redo, st);
    if (e != cudaSuccess) return cuda_fail(e, "overflow_latch_launch");
    timer_end(x, st, t0, FI8_KERNEL_REDO, 0.0);
    x->last_launches++;
    return launch_bin_popcount(b, d_q, M, cand, d_keys, sorted, st, x->d_redo);
  }
  return launch_bin_popcount(b, d_q, M, cand, d_keys, sorted, st);
}

static int launch_bin_rerank(fi8_bin* b, const float* d_q, int32_t M, const uint64_t* d_short, int32_t cand,
                             int32_t k, uint64_t* d_keys, cudaStream_t st) {
  fi8_index* x = b->ix;
  if (cand > kRerankMaxCand || k > cand || k > kMergeMaxK)
    return fail(FI8_ERR_DECLINED, "gpu: rerank declined (cand=%d k=%d)", cand, k);
  int rc;
  if ((rc = ensure_device(&b->d_parts, &b->parts_cap, (size_t)rerank_parts(cand) * M * k, "rerank parts")) !=
      FI8_OK)
    return rc;
  cudaEvent_t t0 = timer_begin(x, st);
  cudaError_t e = rerank_launch(d_q, M, x->dim, x->dpad, x->d_codes, x->d_scales, x->n, x->id_base, d_short, cand,
                                k, b->d_parts, d_keys, st);
  if (e != cudaSuccess) return cuda_fail(e, "rerank_launch");
  timer_end(x, st, t0, FI8_KERNEL_RERANK, (double)M * cand * (x->dpad + 4 + 8));
  x->last_launches += 2;
  return FI8_OK;
}

extern "C" {

int fi8_bin_index_create(fi8_ctx* ctx, const uint64_t* codes, int32_t words, const float* center,
                         const int8_t* i8, const float* scales, int64_t n, int32_t dim, int32_t overquery,
                         int64_t id_base, fi8_bin** out) {
  if (!out) return fail(FI8_ERR_ARG, "fi8_bin_index_create: null out");
  *out = nullptr;
  if (!ctx || !codes) return fail(FI8_ERR_ARG, "fi8_bin_index_create: null argument");
  if (dim <= 0 || words != (dim + 63) / 64)  // linalg.PackedWords
    return fail(FI8_ERR_ARG, "fi8_bin_index_create: words=%d does not match dim %d", words, dim);
  const int32_t wpad = (words + 1) / 2 * 2;
  if (wpad * 8 > kScanMaxDpad)
    return fail(FI8_ERR_DECLINED, "fi8_bin_index_create: dim %d exceeds the supported packed width", dim);
  fi8_index* ix = nullptr;
  int rc = fi8_index_create(ctx, i8, scales, n, dim, id_base, &ix);
  if (rc != FI8_OK) return rc;
  fi8_bin* b = new (std::nothrow) fi8_bin;
  if (!b) {
    fi8_index_destroy(ix);
    return fail(FI8_ERR_OOM, "fi8_bin_index_create: host allocation");
  }
  b->ix = ix;
  b->words = words;
  b->wpad = wpad;
  b->over = overquery < 1 ? 1 : overquery;
  DeviceGuard g(ix->device);
  const size_t pitch = (size_t)wpad * 8;
  PinnedStager stage;
  cudaError_t e = stage.init();
  if (e == cudaSuccess) e = cudaMalloc(&b->d_bits, (size_t)ix->n_alloc * pitch);
  if (e == cudaSuccess) e = cudaMemsetAsync(b->d_bits, 0, (size_t)ix->n_alloc * pitch, ix->stream);
  if (e == cudaSuccess) e = stage.put_rows(b->d_bits, pitch, codes, (size_t)words * 8, (size_t)words * 8, n, ix->stream);
  if (e == cudaSuccess) e = stage.finish();
  if (e == cudaSuccess && center) {
    e = cudaMalloc(&b->d_center, (size_t)dim * sizeof(float));
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(b->d_center, center, (size_t)dim * sizeof(float), cudaMemcpyHostToDevice, ix->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ix->stream);
  if (e != cudaSuccess) {
    rc = cuda_fail(e, "gpu: binary index upload failed");
    fi8_bin_index_destroy(b);
    return rc;
  }
  *out = b;
  return FI8_OK;
}

int fi8_bin_index_create_empty(fi8_ctx* ctx, int64_t n, int32_t dim, int32_t words, const float* center,
                               int32_t overquery, int64_t id_base, fi8_bin** out) {
  if (!out) return fail(FI8_ERR_ARG, "fi8_bin_index_create_empty: null out");
  *out = nullptr;
  if (!ctx) return fail(FI8_ERR_ARG, "fi8_bin_index_create_empty: null ctx");
  if (dim <= 0 || words != (dim + 63) / 64)  // linalg.PackedWords
    return fail(FI8_ERR_ARG, "fi8_bin_index_create_empty: words=%d does not match dim %d", words, dim);
  const int32_t wpad = (words + 1) / 2 * 2;
  if (wpad * 8 > kScanMaxDpad)
    return fail(FI8_ERR_DECLINED, "fi8_bin_index_create_empty: dim %d exceeds the supported packed width", dim);
  fi8_index* ix = nullptr;
  int rc = fi8_index_create_empty(ctx, n, dim, id_base, &ix);
  if (rc != FI8_OK) return rc;
  fi8_bin* b = new (std::nothrow) fi8_bin;
  if (!b) {
    fi8_index_destroy(ix);
    return fail(FI8_ERR_OOM, "fi8_bin_index_create_empty: host allocation");
  }
  b->ix = ix;
  b->words = words;
  b->wpad = wpad;
  b->over = overquery < 1 ? 1 : overquery;
  DeviceGuard g(ix->device);
  const size_t bytes = (size_t)ix->n_alloc * wpad * 8;
  cudaError_t e = cudaMalloc(&b->d_bits, bytes);
  if (e == cudaSuccess) e = cudaMemsetAsync(b->d_bits, 0, bytes, ix->stream);
  if (e == cudaSuccess && center) {
    e = cudaMalloc(&b->d_center, (size_t)dim * sizeof(float));
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(b->d_center, center, (size_t)dim * sizeof(float), cudaMemcpyHostToDevice, ix->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ix->stream);
  if (e != cudaSuccess) {
    rc = cuda_fail(e, "gpu: binary index allocation failed");
    fi8_bin_index_destroy(b);
    return rc;
  }
  *out = b;
  return FI8_OK;
}

int fi8_bin_upload_rows(fi8_bin* b, int64_t row0, const uint64_t* codes, const int8_t* i8, const float* scales,
                        int64_t rows) {
  if (!b) return fail(FI8_ERR_ARG, "fi8_bin_upload_rows: null index");
  if (rows == 0) return FI8_OK;
  fi8_index* x = b->ix;
  if (rows < 0 || row0 < 0 || row0 + rows > x->n || !codes || !i8 || !scales)
    return fail(FI8_ERR_ARG, "fi8_bin_upload_rows: rows [%lld, %lld) outside [0, %lld) or null data",
                (long long)row0, (long long)(row0 + rows), (long long)x->n);
  std::lock_guard<std::mutex> lk(x->mu);
  DeviceGuard g(x->device);
  if (b->d_sign)
    return fail(FI8_ERR_ARG, "fi8_bin_upload_rows: the tensor-core prefilter's sign rows are built; "
                             "upload every row first");
  if (!x->up_stage) {
    x->up_stage = new (std::nothrow) PinnedStager;
    if (!x->up_stage) return fail(FI8_ERR_OOM, "fi8_bin_upload_rows: host allocation");
    cudaError_t e = x->up_stage->init();
    if (e != cudaSuccess) {
      delete x->up_stage;
      x->up_stage = nullptr;
      return cuda_fail(e, "gpu: pinned staging buffers");
    }
  }
  const size_t wb = (size_t)b->words * 8;
  cudaError_t e = x->up_stage->put_rows(x->d_codes + (size_t)row0 * x->dpad, x->dpad, i8, x->dim, x->dim, rows,
                                        x->stream);
  if (e == cudaSuccess) e = x->up_stage->put_rows(x->d_scales + row0, 4, scales, 4, 4, rows, x->stream);
  if (e == cudaSuccess)
    e = x->up_stage->put_rows(b->d_bits + (size_t)row0 * b->wpad, (size_t)b->wpad * 8, codes, wb, wb, rows,
                              x->stream);
  if (e != cudaSuccess) return cuda_fail(e, "gpu: device upload failed");
  return FI8_OK;
}

int fi8_bin_upload_finish(fi8_bin* b) {
  if (!b) return fail(FI8_ERR_ARG, "fi8_bin_upload_finish: null index");
  return fi8_index_upload_finish(b->ix);
}

int fi8_bin_index_create_f32(fi8_ctx* ctx, const float* vecs, const uint8_t* valid, int64_t n, int32_t dim,
                             int32_t overquery, int32_t centered, const float* center, int64_t id_base,
                             fi8_bin** out) {
  if (!out) return fail(FI8_ERR_ARG, "fi8_bin_index_create_f32: null out");
  *out = nullptr;
  if (n > 0 && dim > 0 && !vecs) return fail(FI8_ERR_ARG, "fi8_bin_index_create_f32: null vectors");
  fi8_index* ix = nullptr;
  int rc = index_alloc(ctx, n, dim, id_base, "fi8_bin_index_create_f32", &ix);
  if (rc != FI8_OK) return rc;
  fi8_bin* b = new (std::nothrow) fi8_bin;
  if (!b) {
    index_free(ix);
    return fail(FI8_ERR_OOM, "fi8_bin_index_create_f32: host allocation");
  }
  b->ix = ix;
  b->words = (dim + 63) / 64;
  b->wpad = (b->words + 1) / 2 * 2;
  b->over = overquery < 1 ? 1 : overquery;
  if (b->wpad * 8 > kScanMaxDpad) {
    fi8_bin_index_destroy(b);
    return fail(FI8_ERR_DECLINED, "fi8_bin_index_create_f32: dim %d exceeds the supported packed width", dim);
  }
  DeviceGuard g(ix->device);
  cudaStream_t st = ix->stream;
  const int64_t chunk = std::min<int64_t>(n, build_chunk_rows(dim));
  float* d_v = nullptr;
  uint8_t* d_valid = nullptr;
  double* d_acc = nullptr;
  PinnedStager stage;
  cudaError_t e = stage.init();
  if (e == cudaSuccess) e = cudaMalloc(&b->d_bits, (size_t)ix->n_alloc * b->wpad * 8);
  if (e == cudaSuccess) e = cudaMemsetAsync(b->d_bits, 0, (size_t)ix->n_alloc * b->wpad * 8, st);
  if (e == cudaSuccess) e = cudaMalloc(&d_v, (size_t)chunk * dim * sizeof(float));
  if (e == cudaSuccess && valid) e = cudaMalloc(&d_valid, (size_t)chunk);
  // The centre: given, computed here (newBinaryPrefilter's float64 mean over
  // the valid rows, prefilter.go:64-85), or none (uncentred, or no valid row).
  const bool compute = centered && !center;
  int64_t used = 0;
  if (compute) {
    if (valid)
      for (int64_t r = 0; r < n; r++) used += valid[r] != 0;
    else
      used = n;
  }
  const bool has_center = centered && (center || used > 0);
  if (e == cudaSuccess && has_center) e = cudaMalloc(&b->d_center, (size_t)dim * sizeof(float));
  if (e == cudaSuccess && has_center && center)
    e = cudaMemcpyAsync(b->d_center, center, (size_t)dim * sizeof(float), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && compute && used > 0) {
    e = cudaMalloc(&d_acc, (size_t)dim * sizeof(double));
    if (e == cudaSuccess) e = cudaMemsetAsync(d_acc, 0, (size_t)dim * sizeof(double), st);
  }
  // pass 1: int8 rows (and the column sums, when the centre is computed here);
  // pass 2, or the same pass when the centre is known: the sign codes
  for (int pass = 0; pass < 2 && e == cudaSuccess; pass++) {
    const bool pack_now = (pass == 0) != (compute && used > 0);
    if (pass == 1 && !pack_now) break;
    if (pass == 1 && compute && used > 0) e = center_launch(d_acc, dim, used, b->d_center, st);
    const size_t rb = (size_t)dim * sizeof(float);
    for (int64_t r0 = 0; e == cudaSuccess && r0 < n; r0 += chunk) {
      const int64_t rows = std::min(chunk, n - r0);
      // stream order keeps the next chunk's copies behind this chunk's kernels
      e = stage.put_rows(d_v, rb, vecs + (size_t)r0 * dim, rb, rb, rows, st);
      if (e == cudaSuccess && valid) e = stage.put_rows(d_valid, 1, valid + r0, 1, 1, rows, st);
      if (e == cudaSuccess && pass == 0)
        e = quantize_rows_launch(d_v, rows, dim, ix->dpad, ix->d_codes + (size_t)r0 * ix->dpad, ix->d_scales + r0,
                                 st);
      if (e == cudaSuccess && pass == 0 && compute && used > 0)
        e = column_sum_launch(d_v, rows, dim, valid ? d_valid : nullptr, d_acc, st);
      if (e == cudaSuccess && pack_now)
        e = pack_rows_launch(d_v, rows, dim, has_center ? b->d_center : nullptr, valid ? d_valid : nullptr, b->wpad,
                             b->d_bits + (size_t)r0 * b->wpad, st);
    }
  }
  if (e == cudaSuccess) e = stage.finish();
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  cudaFree(d_v);
  cudaFree(d_valid);
  cudaFree(d_acc);
  if (e != cudaSuccess || (rc = index_finish(ix)) != FI8_OK) {
    if (e != cudaSuccess) rc = cuda_fail(e, "gpu: binary device build failed");
    fi8_bin_index_destroy(b);
    return rc;
  }
  *out = b;
  return FI8_OK;
}

int fi8_bin_center(fi8_bin* b, float* out, int32_t* has_center) {
  if (!b || !out || !has_center) return fail(FI8_ERR_ARG, "fi8_bin_center: null argument");
  std::lock_guard<std::mutex> lk(b->ix->mu);
  DeviceGuard g(b->ix->device);
  *has_center = b->d_center ? 1 : 0;
  if (b->d_center)
    FI8_CUDA(cudaMemcpy(out, b->d_center, (size_t)b->ix->dim * sizeof(float), cudaMemcpyDeviceToHost), "D2H center");
  return FI8_OK;
}

int fi8_bin_read_codes(fi8_bin* b, uint64_t* codes) {
  if (!b || !codes) return fail(FI8_ERR_ARG, "fi8_bin_read_codes: null argument");
  std::lock_guard<std::mutex> lk(b->ix->mu);
  DeviceGuard g(b->ix->device);
  FI8_CUDA(cudaMemcpy2D(codes, (size_t)b->words * 8, b->d_bits, (size_t)b->wpad * 8, (size_t)b->words * 8,
                        (size_t)b->ix->n, cudaMemcpyDeviceToHost),
           "D2H codes");
  return FI8_OK;
}

int fi8_bin_index_destroy(fi8_bin* b) {
  if (!b) return FI8_OK;
  if (b->ix) {
    {
      std::lock_guard<std::mutex> lk(b->ix->mu);
    }
    DeviceGuard g(b->ix->device);
    cudaStreamSynchronize(b->ix->stream);
    cudaFree(b->d_bits);
    cudaFree(b->d_center);
    cudaFree(b->d_qbits);
    cudaFree(b->d_dist);
    cudaFree(b->d_hist);
    cudaFree(b->d_counts);
    cudaFree(b->d_parts);
    cudaFree(b->d_short);
    cudaFree(b->d_sign);
    fi8_index_destroy(b->ix);
  }
  delete b;
  return FI8_OK;
}

int fi8_bin_set_tensor_prefilter(fi8_bin* b, int32_t min_batch) {
  if (!b || min_batch < 0) return fail(FI8_ERR_ARG, "fi8_bin_set_tensor_prefilter: bad arguments");
  fi8_index* x = b->ix;
  std::lock_guard<std::mutex> lk(x->mu);
  DeviceGuard g(x->device);
  FI8_CUDA(cudaStreamSynchronize(x->stream), "sync");
  if (min_batch == 0) {
    cudaFree(b->d_sign);
    b->d_sign = nullptr;
    b->tensor_min_m = 0;
    return FI8_OK;
  }
  if (!b->d_sign) {
    FI8_CUDA(cudaMalloc(&b->d_sign, (size_t)x->n_alloc * x->dpad), "gpu: sign rows allocation");
    cudaError_t e = sign_rows_launch(b->d_bits, x->n, x->n_alloc, b->wpad, x->dim, x->dpad, b->d_sign, x->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(x->stream);
    if (e == cudaSuccess && !make_tmap_i8(&b->tmS, b->d_sign, (uint64_t)x->n_alloc, (uint64_t)x->dpad,
                                          (uint32_t)kGemmBN))
      e = cudaErrorInvalidValue;
    if (e == cudaSuccess)
      b->has_tmS2 = make_tmap_i8(&b->tmS2, b->d_sign, (uint64_t)x->n_alloc, (uint64_t)x->dpad, (uint32_t)(kGemmBN / 2));
    if (e != cudaSuccess) {
      cudaFree(b->d_sign);
      b->d_sign = nullptr;
      return cuda_fail(e, "gpu: sign rows build failed");
    }
  }
  b->tensor_min_m = min_batch;
  return FI8_OK;
}

int fi8_bin_index_handle(fi8_bin* b, fi8_index** out) {
  if (!b || !out) return fail(FI8_ERR_ARG, "fi8_bin_index_handle: null argument");
  *out = b->ix;
  return FI8_OK;
}

int fi8_bin_query_topk(fi8_bin* b, const float* q, int32_t M, int32_t k, int32_t* out_idx, float* out_score) {
  return fi8_bin_query_topk_keep(b, q, M, k, nullptr, 0, out_idx, out_score);
}

int fi8_bin_query_topk_keep(fi8_bin* b, const float* q, int32_t M, int32_t k, const uint64_t* keep, int64_t nbits,
                            int32_t* out_idx, float* out_score) {
  if (!b) return fail(FI8_ERR_ARG, "fi8_bin_query_topk: null index");
  if (M == 0) return FI8_OK;
  if (M < 0 || !q || !out_idx || !out_score) return fail(FI8_ERR_ARG, "fi8_bin_query_topk: bad arguments");
  fi8_index* x = b->ix;
  // k <= 0 and k >= n return the whole corpus in the reference
  // (flat_binary_i8.go:95-97 -> FlatI8.query); the device declines them.
  if (k <= 0 || (int64_t)k >= x->n)
    return fail(FI8_ERR_DECLINED, "gpu: binary TopK declined (k=%d n=%lld)", k, (long long)x->n);
  const int64_t cand = (int64_t)k * b->over;
  std::lock_guard<std::mutex> lk(x->mu);
  DeviceGuard g(x->device);
  int rc;
  const uint64_t* d_keep = nullptr;
  if ((rc = stage_keep(x, keep, nbits, &d_keep)) != FI8_OK) return rc;
  KeepScope ks(x, d_keep, nbits);
  if ((rc = ensure_device(&x->d_q, &x->d_q_cap, (size_t)M * x->dim, "staging q")) != FI8_OK) return rc;
  FI8_CUDA(cudaMemcpyAsync(x->d_q, q, (size_t)M * x->dim * sizeof(float), cudaMemcpyHostToDevice, x->stream),
           "H2D queries");
  if (cand >= x->n) {
    // the candidate set is the whole corpus: FlatI8's exact scan
    // (flat_binary_i8.go:95-97)
    if ((rc = topk_staged(x, M, k)) != FI8_OK) return rc;
    return fi8_keys_unpack(x->h_keys, (int64_t)M * k, out_idx, out_score);
  }
  const size_t nk = (size_t)M * k;
  x->last_launches = 0;
  if ((rc = ensure_device(&b->d_short, &b->short_cap, (size_t)M * cand, "shortlist")) != FI8_OK) return rc;
  if ((rc = ensure_device(&x->d_keys, &x->d_keys_cap, nk, "staging keys")) != FI8_OK) return rc;
  if ((rc = ensure_host(&x->h_keys, &x->h_keys_cap, nk, "pinned keys")) != FI8_OK) return rc;
  if (cand > kBinMaxCand)
    return fail(FI8_ERR_DECLINED, "gpu: binary TopK declined (cand=%lld beyond %d)", (long long)cand, kBinMaxCand);
  // (a tensor-core shortlist that dropped candidates is redone on the
  // device inside launch_bin_prefilter)
  if ((rc = launch_bin_prefilter(b, x->d_q, M, (int32_t)cand, b->d_short, false, x->stream)) != FI8_OK) return rc;
  if ((rc = launch_bin_rerank(b, x->d_q, M, b->d_short, (int32_t)cand, k, x->d_keys, x->stream)) != FI8_OK)
    return rc;
  FI8_CUDA(cudaMemcpyAsync(x->h_keys, x->d_keys, nk * sizeof(uint64_t), cudaMemcpyDeviceToHost, x->stream),
           "D2H keys");
  FI8_CUDA(cudaMemcpyAsync(x->h_err, x->d_err, sizeof(unsigned int), cudaMemcpyDeviceToHost, x->stream),
           "D2H err");
  FI8_CUDA(cudaStreamSynchronize(x->stream), "sync");
  if ((rc = check_device_error(x)) != FI8_OK) return rc;
  return fi8_keys_unpack(x->h_keys, (int64_t)nk, out_idx, out_score);
}

int fi8_bin_prefilter_async_keep(fi8_bin* b, const float* d_q, int32_t M, int32_t cand, const uint64_t* d_keep,
                                 int64_t nbits, uint64_t* d_keys, int32_t sorted, void* stream) {
  if (!b) return fail(FI8_ERR_ARG, "fi8_bin_prefilter_async: null index");
  if (M == 0) return FI8_OK;
  if (M < 0 || !d_q || !d_keys || nbits < 0) return fail(FI8_ERR_ARG, "fi8_bin_prefilter_async: bad arguments");
  if (cand <= 0) return fail(FI8_ERR_DECLINED, "gpu: binary prefilter declined (cand=%d)", cand);
  std::lock_guard<std::mutex> lk(b->ix->mu);
  DeviceGuard g(b->ix->device);
  KeepScope ks(b->ix, d_keep, nbits);
  b->ix->last_launches = 0;
  return launch_bin_prefilter(b, d_q, M, cand, d_keys, sorted != 0, static_cast<cudaStream_t>(stream));
}

int fi8_bin_prefilter_async(fi8_bin* b, const float* d_q, int32_t M, int32_t cand, uint64_t* d_keys, int32_t sorted,
                            void* stream) {
  return fi8_bin_prefilter_async_keep(b, d_q, M, cand, nullptr, 0, d_keys, sorted, stream);
}

int fi8_bin_rerank_async(fi8_bin* b, const float* d_q, int32_t M, const uint64_t* d_short, int32_t cand, int32_t k,
                         uint64_t* d_keys, void* stream) {
  if (!b) return fail(FI8_ERR_ARG, "fi8_bin_rerank_async: null index");
  if (M == 0) return FI8_OK;
  if (M < 0 || !d_q || !d_short || !d_keys || cand <= 0)
    return fail(FI8_ERR_ARG, "fi8_bin_rerank_async: bad arguments");
  if (k <= 0) return fail(FI8_ERR_DECLINED, "gpu: rerank declined (k=%d)", k);
  std::lock_guard<std::mutex> lk(b->ix->mu);
  DeviceGuard g(b->ix->device);
  b->ix->last_launches = 0;
  return launch_bin_rerank(b, d_q, M, d_short, cand, k, d_keys, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

extern "C" int fi8_gemm_plan(int64_t n, int32_t M, int32_t k, int64_t* out_bounds, int32_t max_bounds,
                             int32_t* count) {
  if (n <= 0 || M <= 0 || k <= 0 || !out_bounds || !count || max_bounds < 2)
    return fail(FI8_ERR_ARG, "fi8_gemm_plan: bad arguments");
  std::vector<GemmLevel> ranges;
  plan_ranges(n, M, k, gemm_cap(M), &ranges);
  *count = (int32_t)ranges.size();
  if ((int64_t)ranges.size() + 1 > max_bounds)
    return fail(FI8_ERR_ARG, "fi8_gemm_plan: %zu ranges need %zu bounds", ranges.size(), ranges.size() + 1);
  for (size_t i = 0; i < ranges.size(); i++) out_bounds[i] = ranges[i].row_lo;
  out_bounds[ranges.size()] = ranges.back().row_hi;
  return FI8_OK;
}
