// fi8_binary.cu -- the two small kernels of the FlatBinaryI8 device path.
//
// Reference semantics (ann/flat_binary_i8.go:86-153, flat_binary_prefilter.go):
// the query is centred and packed to sign bits (centered :100-108,
// PackSignBitsRow linalg/hamming.go:28-37); the prefilter keeps the cand rows
// nearest in Hamming distance, ties by ascending id (prefilterHist :145-216);
// the rerank scores those rows with FlatI8's W8A8 and keeps the best k under
// (score desc, index asc) with NaN rejected (rerank :122-153).
//
// The prefilter's "smallest t with cum >= cand, every d < t, then the first
// budget rows with d == t in id order" is exactly the cand smallest rows under
// (distance asc, id asc), so the scan kernel's binary mode selects it as a
// top-K over keys of (-distance, id). The rerank kernel here scores the
// shortlist and sorts it in shared memory.
#include "fi8_binary.cuh"
#include "fi8_device.cuh"
#include "fi8_select.cuh"

namespace fi8 {

namespace {

constexpr int kRerankThreads = 512;

__global__ void __launch_bounds__(256) binary_prep_kernel(const float* q, int d, const float* center, int wpad,
                                                          uint64_t* qbits) {
  const int y = blockIdx.x;
  const float* row = q + (size_t)y * d;
  for (int w = threadIdx.x; w < wpad; w += blockDim.x) {
    uint64_t bits = 0;
    const int i0 = w * 64;
    for (int b = 0; b < 64 && i0 + b < d; b++) {
      float x = row[i0 + b];
      if (center) x = __fsub_rn(x, center[i0 + b]);
      if (x >= 0.0f) bits |= 1ull << b;  // NaN compares false: bit clear
    }
    qbits[(size_t)y * wpad + w] = bits;
  }
}

// One CTA per query. An 8-lane quarter-warp scores one shortlist row (16-byte
// chunks, dp4a, reduced over the quarter); survivors' keys go to a shared
// buffer that is then sorted.
__global__ void __launch_bounds__(kRerankThreads, 1)
    rerank_kernel(const float* q, int d, int dpad, const int8_t* codes, const float* scales, int64_t n,
                  uint32_t id_base, const uint64_t* shortlist, int cand, int candp, int k, uint64_t* out) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float s_red[kRerankThreads / 32];
  __shared__ float s_qscale;
  __shared__ int s_count;
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem);               // [candp]
  int8_t* q_s = reinterpret_cast<int8_t*>(smem + (size_t)candp * 8);  // [dpad]
  const int y = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  constexpr int bar = 1;

  // quantize the query (quant.go:43-71, all-zero -> scale 0)
  const float* qy = q + (size_t)y * d;
  float m = 0.0f;
  for (int i = tid; i < d; i += kRerankThreads) m = absmax_step(m, qy[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = absmax_combine(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) s_red[warp] = m;
  if (tid == 0) s_count = 0;
  __syncthreads();
  if (tid == 0) {
    float mm = 0.0f;
    for (int w = 0; w < kRerankThreads / 32; w++) mm = absmax_combine(mm, s_red[w]);
    s_red[0] = mm;
  }
  __syncthreads();
  const float maxabs = s_red[0];
  if (maxabs == 0.0f) {
    for (int i = tid; i < dpad; i += kRerankThreads) q_s[i] = 0;
    if (tid == 0) s_qscale = 0.0f;
  } else {
    const float sc = __fdiv_rn(maxabs, 127.0f);
    const float inv = __fdiv_rn(1.0f, sc);
    for (int i = tid; i < dpad; i += kRerankThreads) q_s[i] = i < d ? quant_code(qy[i], inv) : (int8_t)0;
    if (tid == 0) s_qscale = sc;
  }
  __syncthreads();
  const float qscale = s_qscale;

  const int lane8 = lane & 7;
  const int slot = tid >> 3;  // quarter-warp index
  constexpr int kSlots = kRerankThreads / 8;
  const int chunks = dpad >> 4;
  const uint64_t* sl = shortlist + (size_t)y * cand;
  for (int e0 = 0; e0 < cand; e0 += kSlots) {
    const int e = e0 + slot;
    int64_t local = -1;
    uint32_t gid = 0;
    if (e < cand) {
      const uint64_t key = sl[e];
      if (key != kEmptyKey) {
        gid = (uint32_t)key_index(key);
        const int64_t l = (int64_t)gid - (int64_t)id_base;
        if (l >= 0 && l < n) local = l;
      }
    }
    int acc = 0;
    if (local >= 0) {
      const int4* rowp = reinterpret_cast<const int4*>(codes + (size_t)local * dpad);
      const int4* qp = reinterpret_cast<const int4*>(q_s);
      for (int c = lane8; c < chunks; c += 8) {
        const int4 a = __ldg(rowp + c), b = qp[c];
        acc = __dp4a(a.x, b.x, acc);
        acc = __dp4a(a.y, b.y, acc);
        acc = __dp4a(a.z, b.z, acc);
        acc = __dp4a(a.w, b.w, acc);
      }
    }
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane8 == 0 && local >= 0) {
      const float score = w8a8_score(acc, qscale, scales[local]);
      if (score == score) buf[atomicAdd(&s_count, 1)] = make_key(score, gid);
    }
  }
  __syncthreads();
  const int cnt = s_count;
  for (int i = cnt + tid; i < candp; i += kRerankThreads) buf[i] = kEmptyKey;
  named_sync(bar, kRerankThreads);
  group_sort_desc<kRerankThreads>(buf, candp, tid, bar);
  for (int i = tid; i < k; i += kRerankThreads) out[(size_t)y * k + i] = i < cnt ? buf[i] : kEmptyKey;
}

int pow2_ceil(int x) {
  int p = 2;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace

cudaError_t binary_prep_launch(const float* q, int32_t M, int32_t d, const float* center, int32_t wpad,
                               uint64_t* qbits, cudaStream_t stream) {
  if (M <= 0 || d <= 0 || wpad * 64 < d) return cudaErrorInvalidValue;
  binary_prep_kernel<<<M, 256, 0, stream>>>(q, d, center, wpad, qbits);
  return cudaGetLastError();
}

cudaError_t rerank_launch(const float* q, int32_t M, int32_t d, int32_t dpad, const int8_t* codes,
                          const float* scales, int64_t n, uint32_t id_base, const uint64_t* shortlist,
                          int32_t cand, int32_t k, uint64_t* out, cudaStream_t stream) {
  if (M <= 0 || cand <= 0 || cand > kRerankMaxCand || k <= 0 || dpad % 16 != 0) return cudaErrorInvalidValue;
  const int candp = pow2_ceil(cand > k ? cand : k);
  const size_t smem = (size_t)candp * 8 + (size_t)dpad;
  cudaError_t e = cudaFuncSetAttribute(rerank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)((size_t)kRerankMaxCand * 8 + 2048));
  if (e != cudaSuccess) return e;
  rerank_kernel<<<M, kRerankThreads, smem, stream>>>(q, d, dpad, codes, scales, n, id_base, shortlist, cand, candp,
                                                      k, out);
  return cudaGetLastError();
}

}  // namespace fi8
