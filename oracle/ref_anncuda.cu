// ref_anncuda.cu -- TEST INFRASTRUCTURE: the reference's own CUDA kernels
// (gpu/anncuda/gemv_w8a8.cu, compiled for sm_100a from the reference source
// tree, which the build puts on the include path) behind a small C launcher,
// so tests and the benchmark can run the device path this library replaces on
// the same B200 and compare with it.
//
// Nothing of the reference is copied here. The launcher restates the host
// side of gpu/anncuda/backend.go that picks and sizes those launches:
//   * launchBatch (backend.go:675-712): gemv_w8a8 for one query, n*16 threads
//     in 256-thread blocks; otherwise batchPlan (:715-720) -- batch8 (8 lanes,
//     8-query tiles) up to 8 queries, batch16 (4 lanes, 16-query tiles) above
//     -- with grid (batchGridX(ceil(n*lanes/256), planes, sm), planes) and
//     qtile*dim bytes of dynamic shared memory;
//   * batchGridX (:512-527): full/8 blocks, at least ceil(4*sm/planes), at
//     most full;
//   * launchTopK (:468-510) with topkPlan (:372-379) and topkSplitParts
//     (:400-415): k above 64 runs topk_rows (k passes, one 256-thread block per
//     query); otherwise, when the split pays (M below the SM count), topk_split
//     over min(n/4096, 1024/M) parts then topk_merge, else topk_rows_r<w>.
// Scalars travel as 1-element device buffers, as the reference binds them.
// The queries are quantized on the host by the caller (the reference's
// quantizeRowInt8, backend.go:270-298), so the inputs here are int8 rows and
// their scales.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <new>

#include "gemv_w8a8.cu"  // the reference kernels, from the reference source tree

namespace {

constexpr int kBlock = 256;           // batchBlock, topkBlockThreads
constexpr int kGemvLanes = 16;        // gemvLanes
constexpr int kSplitChunk = 4096;     // topkSplitChunk
constexpr int kSplitMaxBlocks = 1024; // topkSplitMaxBlocks
const int kWidths[4] = {8, 16, 32, 64};

int topk_plan(uint32_t k) {
  for (int i = 0; i < 4; i++)
    if ((int)k <= kWidths[i]) return i;
  return -1;
}

int split_parts(uint32_t M, uint32_t n, int sm) {
  if ((int)M >= sm) return 1;
  int parts = (int)(n / kSplitChunk);
  const int cap = kSplitMaxBlocks / (int)M;
  if (parts > cap) parts = cap;
  return parts < 1 ? 1 : parts;
}

uint32_t batch_grid_x(uint64_t full, int planes, int sm) {
  uint64_t gx = full / 8;
  const uint64_t lo = (uint64_t)(4 * sm + planes - 1) / (uint64_t)planes;
  if (gx < lo) gx = lo;
  if (gx > full) gx = full;
  if (gx < 1) gx = 1;
  return (uint32_t)gx;
}

}  // namespace

// One prepared query shape: the scalar buffers and the split scratch.
struct ref_plan {
  uint32_t n, dim, M, k;
  int sm;
  unsigned int* d_scalars = nullptr;  // [0] n, [1] dim, [2] M, [3] k, [4] parts*k
  int parts = 1;
  int width = -1;
  int32_t* part_idx = nullptr;
  float* part_val = nullptr;
};

extern "C" {

// Prepare a TopKBatch of M queries with k over an index of n rows of dim
// bytes on the current device (sm = its SM count).
int ref_plan_create(uint32_t n, uint32_t dim, uint32_t M, uint32_t k, int sm, ref_plan** out) {
  *out = nullptr;
  if (n == 0 || dim == 0 || M == 0 || k == 0 || sm <= 0) return 1;
  ref_plan* p = new (std::nothrow) ref_plan;
  if (!p) return 2;
  p->n = n;
  p->dim = dim;
  p->M = M;
  p->k = k;
  p->sm = sm;
  p->width = topk_plan(k);
  p->parts = split_parts(M, n, sm);
  unsigned int h[5] = {n, dim, M, k, (unsigned int)(p->parts * k)};
  cudaError_t e = cudaMalloc(&p->d_scalars, sizeof(h));
  if (e == cudaSuccess) e = cudaMemcpy(p->d_scalars, h, sizeof(h), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && p->parts > 1 && p->width >= 0) {
    const size_t slots = (size_t)M * p->parts * k;
    e = cudaMalloc(&p->part_idx, slots * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMalloc(&p->part_val, slots * sizeof(float));
  }
  if (e != cudaSuccess) {
    cudaFree(p->d_scalars);
    cudaFree(p->part_idx);
    cudaFree(p->part_val);
    delete p;
    return 3;
  }
  *out = p;
  return 0;
}

int ref_plan_destroy(ref_plan* p) {
  if (!p) return 0;
  cudaFree(p->d_scalars);
  cudaFree(p->part_idx);
  cudaFree(p->part_val);
  delete p;
  return 0;
}

// launchBatch: scores [M][n] of the int8 queries qi8 [M][dim] (scales qscale
// [M]) against codes [n][dim] / scales [n].
int ref_score_launch(ref_plan* p, const int8_t* codes, const float* scales, const int8_t* qi8,
                     const float* qscale, float* scores, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned int* N = p->d_scalars;
  const unsigned int* K = p->d_scalars + 1;
  const unsigned int* M = p->d_scalars + 2;
  const signed char* c = reinterpret_cast<const signed char*>(codes);
  const signed char* q = reinterpret_cast<const signed char*>(qi8);
  if (p->M == 1) {
    const uint64_t threads = (uint64_t)p->n * kGemvLanes;
    gemv_w8a8<<<(unsigned)((threads + kBlock - 1) / kBlock), kBlock, 0, st>>>(c, q, scales, K, qscale, scores, N);
  } else {
    const bool wide = p->M > 8;
    const int lanes = wide ? 4 : 8, qtile = wide ? 16 : 8;
    const int planes = (int)((p->M + qtile - 1) / qtile);
    const uint64_t full = ((uint64_t)p->n * lanes + kBlock - 1) / kBlock;
    dim3 grid(batch_grid_x(full, planes, p->sm), (unsigned)planes);
    const size_t smem = (size_t)qtile * p->dim;
    if (wide)
      gemv_w8a8_batch16<<<grid, kBlock, smem, st>>>(c, q, scales, K, qscale, scores, N, M);
    else
      gemv_w8a8_batch8<<<grid, kBlock, smem, st>>>(c, q, scales, K, qscale, scores, N, M);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

// launchTopK over scores [M][n] (topk_rows consumes them): idx / val [M][k].
int ref_topk_launch(ref_plan* p, float* scores, int32_t* idx, float* val, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned int* N = p->d_scalars;
  const unsigned int* M = p->d_scalars + 2;
  const unsigned int* K = p->d_scalars + 3;
  const unsigned int* P = p->d_scalars + 4;
  const int w = p->width;
  if (p->parts <= 1 || w < 0) {
    switch (w) {
      case 0: topk_rows_r8<<<p->M, kBlock, 0, st>>>(scores, idx, val, M, N, K); break;
      case 1: topk_rows_r16<<<p->M, kBlock, 0, st>>>(scores, idx, val, M, N, K); break;
      case 2: topk_rows_r32<<<p->M, kBlock, 0, st>>>(scores, idx, val, M, N, K); break;
      case 3: topk_rows_r64<<<p->M, kBlock, 0, st>>>(scores, idx, val, M, N, K); break;
      default: topk_rows<<<p->M, kBlock, 0, st>>>(scores, idx, val, M, N, K); break;
    }
    return cudaGetLastError() == cudaSuccess ? 0 : 4;
  }
  dim3 grid((unsigned)p->parts, p->M);
  switch (w) {
    case 0:
      topk_split_r8<<<grid, kBlock, 0, st>>>(scores, p->part_idx, p->part_val, M, N, K);
      topk_merge_r8<<<p->M, kBlock, 0, st>>>(p->part_idx, p->part_val, idx, val, M, P, K);
      break;
    case 1:
      topk_split_r16<<<grid, kBlock, 0, st>>>(scores, p->part_idx, p->part_val, M, N, K);
      topk_merge_r16<<<p->M, kBlock, 0, st>>>(p->part_idx, p->part_val, idx, val, M, P, K);
      break;
    case 2:
      topk_split_r32<<<grid, kBlock, 0, st>>>(scores, p->part_idx, p->part_val, M, N, K);
      topk_merge_r32<<<p->M, kBlock, 0, st>>>(p->part_idx, p->part_val, idx, val, M, P, K);
      break;
    default:
      topk_split_r64<<<grid, kBlock, 0, st>>>(scores, p->part_idx, p->part_val, M, N, K);
      topk_merge_r64<<<p->M, kBlock, 0, st>>>(p->part_idx, p->part_val, idx, val, M, P, K);
      break;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

// Kernel launches of one TopKBatch (for launch counts).
int ref_plan_launches(const ref_plan* p) { return 1 + ((p->parts <= 1 || p->width < 0) ? 1 : 2); }

}  // extern "C"
