// fi8_binary.cu -- the FlatBinaryI8 device path around the Hamming scan.
//
// Reference semantics (ann/flat_binary_i8.go:86-153, flat_binary_prefilter.go):
// the query is centred and packed to sign bits (centered :100-108,
// PackSignBitsRow linalg/hamming.go:28-37); prefilterHist (:145-216) counts
// the distances of all rows in a (dim+1)-bin histogram, takes the smallest t
// with cum(t) >= cand, and keeps every row with distance < t plus the first
// budget = cand - cum(<t) rows with distance == t in ascending id order; the
// rerank (:122-153) scores those rows with FlatI8's W8A8 and keeps the best k
// under (score desc, index asc), NaN rejected.
//
// Device pipeline per query batch:
//   binary_prep     sign bits of (q - center); zero the histogram
//   scan (binary)   one HBM pass: every row's distance (u16) + histogram
//   shortlist_count per row segment: rows below t, rows at t
//   shortlist_emit  the shortlist as packed keys (-distance, global id), with
//                   the ties at t taken in ascending id across segments
//   rerank          W8A8 scores of the shortlist rows, best k per CTA slice,
//                   then the key merge of the slices
#include "fi8_binary.cuh"
#include "fi8_device.cuh"
#include "fi8_scan.cuh"
#include "fi8_select.cuh"

namespace fi8 {

namespace {

constexpr int kSegThreads = 256;
constexpr int kRowsPerThread = 8;  // one 16-byte load of u16 distances
constexpr int kSegChunk = kSegThreads * kRowsPerThread;
constexpr int kRerankThreads = 512;
constexpr int kRerankRowsPerCta = kRerankThreads / 8;  // one 8-lane group per row

// One CTA per query; thread per dimension, warp ballots build the words.
__global__ void __launch_bounds__(1024) binary_prep_kernel(const float* q, int d, const float* center, int wpad,
                                                           uint64_t* qbits, unsigned int* hist, int nbins,
                                                           const unsigned int* gate) {
  if (gate && *reinterpret_cast<const volatile unsigned int*>(gate) == 0u) return;  // a closed redo gate
  const int y = blockIdx.x;
  const float* row = q + (size_t)y * d;
  uint32_t* out = reinterpret_cast<uint32_t*>(qbits + (size_t)y * wpad);
  const int lane = threadIdx.x & 31;
  for (int base = threadIdx.x - lane; base < wpad * 64; base += blockDim.x) {
    const int i = base + lane;
    bool bit = false;
    if (i < d) {
      float x = row[i];
      if (center) x = __fsub_rn(x, center[i]);
      bit = x >= 0.0f;  // NaN compares false: bit clear
    }
    const uint32_t m = __ballot_sync(0xffffffffu, bit);
    if (lane == 0) out[base >> 5] = m;  // little-endian: bit i%64 of word i/64
  }
  for (int b = threadIdx.x; b < nbins; b += blockDim.x) hist[(size_t)y * nbins + b] = 0u;
}

// Block-wide (kSegThreads) exclusive prefix of v; *total = the sum.
__device__ __forceinline__ long long block_excl_scan64(long long v, long long* total) {
  __shared__ long long s_w[kSegThreads / 32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  long long incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const long long x = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += x;
  }
  if (lane == 31) s_w[w] = incl;
  __syncthreads();
  long long wbase = 0, all = 0;
#pragma unroll
  for (int i = 0; i < kSegThreads / 32; i++) {
    if (i < w) wbase += s_w[i];
    all += s_w[i];
  }
  __syncthreads();
  *total = all;
  return wbase + incl - v;
}

// prefilterHist's cut (prefilter.go:182-189): the smallest t with
// cum(t) + hist[t] >= cand; *lt = cum(t) (rows below t). t = nbins when the
// corpus holds fewer than cand rows (every row is taken). Block-wide.
__device__ void find_cut(const unsigned int* hist, int nbins, int64_t cand, int* t_out, int64_t* lt_out) {
  __shared__ int s_t;
  __shared__ long long s_lt;
  const int tid = threadIdx.x;
  const int per = (nbins + kSegThreads - 1) / kSegThreads;
  const int b0 = tid * per, b1 = min(nbins, b0 + per);
  long long mine = 0;
  for (int b = b0; b < b1; b++) mine += hist[b];
  long long all;
  const long long before = block_excl_scan64(mine, &all);
  if (tid == 0) {
    s_t = nbins;
    s_lt = all;  // fewer than cand rows: all of them are below the cut
  }
  __syncthreads();
  if (before < cand && before + mine >= cand) {  // exactly one thread
    long long cum = before;
    for (int b = b0; b < b1; b++) {
      if (cum + (long long)hist[b] >= cand) {
        s_t = b;
        s_lt = cum;
        break;
      }
      cum += hist[b];
    }
  }
  __syncthreads();
  *t_out = s_t;
  *lt_out = s_lt;
}

__device__ __forceinline__ void seg_bounds(int64_t n, int P, int p, int64_t* lo, int64_t* hi) {
  const int64_t per = ((n + P - 1) / P + kRowsPerThread - 1) / kRowsPerThread * kRowsPerThread;
  *lo = min((int64_t)p * per, n);
  *hi = min(*lo + per, n);
}

// Load 8 consecutive distances starting at row r (rows past hi read as 0xFFFF,
// which is above every cut).
__device__ __forceinline__ void load8(const uint16_t* dist, int64_t r, int64_t hi, uint16_t (&v)[8]) {
  if (r + 8 <= hi) {
    const uint4 w = *reinterpret_cast<const uint4*>(dist + r);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      v[2 * j] = (uint16_t)(ws[j] & 0xFFFFu);
      v[2 * j + 1] = (uint16_t)(ws[j] >> 16);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = (r + j < hi) ? dist[r + j] : (uint16_t)0xFFFFu;
  }
}

// grid (P, M): counts[y][p] = {rows < t, rows == t} of segment p.
__global__ void __launch_bounds__(kSegThreads) shortlist_count_kernel(const uint16_t* dist, int64_t n,
                                                                      int64_t dstride, const unsigned int* hist,
                                                                      int nbins,
                                                                      int64_t cand, int P, unsigned int* counts,
                                                                      const unsigned int* gate) {
  const int p = blockIdx.x, y = blockIdx.y;
  pdl_launch_dependents();
  pdl_wait_prior();  // the distance pass has completed
  if (gate && *reinterpret_cast<const volatile unsigned int*>(gate) == 0u) return;
  int t;
  int64_t lt_all;
  find_cut(hist + (size_t)y * nbins, nbins, cand, &t, &lt_all);
  int64_t lo, hi;
  seg_bounds(n, P, p, &lo, &hi);
  const uint16_t* dy = dist + (size_t)y * dstride;
  unsigned int lt = 0, eq = 0;
  for (int64_t r = lo + (int64_t)threadIdx.x * kRowsPerThread; r < hi; r += kSegChunk) {
    uint16_t v[8];
    load8(dy, r, hi, v);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      lt += v[j] < t;
      eq += v[j] == t;
    }
  }
  __shared__ unsigned int s_lt[kSegThreads / 32], s_eq[kSegThreads / 32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    lt += __shfl_xor_sync(0xffffffffu, lt, off);
    eq += __shfl_xor_sync(0xffffffffu, eq, off);
  }
  if ((threadIdx.x & 31) == 0) {
    s_lt[threadIdx.x >> 5] = lt;
    s_eq[threadIdx.x >> 5] = eq;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int a = 0, b = 0;
    for (int w = 0; w < kSegThreads / 32; w++) {
      a += s_lt[w];
      b += s_eq[w];
    }
    counts[((size_t)y * P + p) * 2] = a;
    counts[((size_t)y * P + p) * 2 + 1] = b;
  }
}

// Exclusive block scan of per-thread counts; returns this thread's offset and
// writes the block total.
__device__ __forceinline__ unsigned int block_excl_scan(unsigned int v, unsigned int* total) {
  __shared__ unsigned int s_w[kSegThreads / 32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const unsigned int x = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += x;
  }
  if (lane == 31) s_w[w] = incl;
  __syncthreads();
  unsigned int wbase = 0, all = 0;
  for (int i = 0; i < kSegThreads / 32; i++) {
    if (i < w) wbase += s_w[i];
    all += s_w[i];
  }
  __syncthreads();
  *total = all;
  return wbase + incl - v;
}

// grid (P, M): write the shortlist keys. Rows below t go to
// [prefix of lower segments' below-t counts + rank]; rows at t take global tie
// ranks in id order and are kept while the rank is below the budget, at
// [all below-t rows + tie rank]. Unfilled slots (fewer than cand rows) are 0.
__global__ void __launch_bounds__(kSegThreads) shortlist_emit_kernel(const uint16_t* dist, int64_t n,
                                                                     int64_t dstride, const unsigned int* hist,
                                                                     int nbins,
                                                                     int64_t cand, int P, const unsigned int* counts,
                                                                     uint32_t id_base, uint64_t* out,
                                                                     const unsigned int* gate) {
  const int p = blockIdx.x, y = blockIdx.y;
  pdl_launch_dependents();
  pdl_wait_prior();  // the segment counts are complete
  if (gate && *reinterpret_cast<const volatile unsigned int*>(gate) == 0u) return;
  int t;
  int64_t lt_all;
  find_cut(hist + (size_t)y * nbins, nbins, cand, &t, &lt_all);
  const int64_t budget = cand - lt_all;
  // lower segments' counts (below t, at t) and all segments' ties at t
  long long a = 0, b = 0, e = 0;
  const unsigned int* cy = counts + (size_t)y * P * 2;
  for (int i = threadIdx.x; i < P; i += kSegThreads) {
    const unsigned int l = cy[2 * i], q = cy[2 * i + 1];
    if (i < p) {
      a += l;
      b += q;
    }
    e += q;
  }
  long long ltp, eqp, eq_all;
  block_excl_scan64(a, &ltp);
  block_excl_scan64(b, &eqp);
  block_excl_scan64(e, &eq_all);
  uint64_t* oy = out + (size_t)y * cand;
  int64_t lo, hi;
  seg_bounds(n, P, p, &lo, &hi);
  const uint16_t* dy = dist + (size_t)y * dstride;
  for (int64_t base = lo; base < hi; base += kSegChunk) {
    const int64_t r = base + (int64_t)threadIdx.x * kRowsPerThread;
    uint16_t v[8];
    unsigned int nl = 0, ne = 0;
    if (r < hi) {
      load8(dy, r, hi, v);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        nl += v[j] < t;
        ne += v[j] == t;
      }
    }
    if (!__syncthreads_or((nl | ne) != 0)) continue;  // the usual chunk: nothing to keep
    unsigned int tl, te;
    unsigned int ol = block_excl_scan(nl, &tl);
    unsigned int oe = block_excl_scan(ne, &te);
    if (nl | ne) {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const uint32_t gid = id_base + (uint32_t)(r + j);
        if (v[j] < t) {
          oy[ltp + ol++] = make_key((float)(-(int)v[j]), gid);
        } else if (v[j] == t) {
          const int64_t er = eqp + oe++;
          if (er < budget) oy[lt_all + er] = make_key((float)(-(int)v[j]), gid);
        }
      }
    }
    ltp += tl;
    eqp += te;
  }
  if (p == 0) {
    const int64_t eq_taken = eq_all < budget ? eq_all : budget;
    for (int64_t i = lt_all + eq_taken + threadIdx.x; i < cand; i += kSegThreads) oy[i] = kEmptyKey;
  }
}

// The sign rows of the tensor-core prefilter: a thread per 16 output bytes
// (16 code bits), one 16-byte store each.
__global__ void __launch_bounds__(256) sign_rows_kernel(const uint64_t* bits, int64_t n, int64_t n_alloc, int wpad,
                                                        int d, int dpad, int8_t* rows) {
  const int chunks = dpad >> 4;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n_alloc * chunks) return;
  const int64_t r = t / chunks;
  const int i0 = (int)(t % chunks) << 4;
  const uint32_t w = r < n ? (uint32_t)(bits[(size_t)r * wpad + (i0 >> 6)] >> (i0 & 63)) & 0xFFFFu : 0u;
  uint32_t o[4];
#pragma unroll
  for (int g = 0; g < 4; g++) {
    uint32_t v = 0;
#pragma unroll
    for (int b = 0; b < 4; b++) {
      const int i = i0 + 4 * g + b;
      const uint32_t byte = (r < n && i < d) ? (((w >> (4 * g + b)) & 1u) ? 0x01u : 0xFFu) : 0u;
      v |= byte << (8 * b);
    }
    o[g] = v;
  }
  reinterpret_cast<uint4*>(rows + (size_t)r * dpad)[i0 >> 4] = make_uint4(o[0], o[1], o[2], o[3]);
}

// One CTA per query: sort its cand keys descending (for the cross-shard merge).
__global__ void __launch_bounds__(1024) sort_keys_kernel(uint64_t* keys, int cand, int candp,
                                                         const unsigned int* gate) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem);
  uint64_t* ky = keys + (size_t)blockIdx.x * cand;
  pdl_launch_dependents();
  pdl_wait_prior();
  if (gate && *reinterpret_cast<const volatile unsigned int*>(gate) == 0u) return;
  for (int i = threadIdx.x; i < candp; i += 1024) buf[i] = i < cand ? ky[i] : kEmptyKey;
  named_sync(1, 1024);
  group_sort_desc<1024>(buf, candp, threadIdx.x, 1);
  for (int i = threadIdx.x; i < cand; i += 1024) ky[i] = buf[i];
}

// grid (P, M): CTA p scores shortlist entries [p*64, p*64 + 64) of query y --
// one 8-lane group per row, 16-byte chunks, dp4a -- and writes its best k
// keys, sorted and 0-padded, to parts[p][y][0..k).
__global__ void __launch_bounds__(kRerankThreads) rerank_kernel(const float* q, int d, int dpad, const int8_t* codes,
                                                               const float* scales, int64_t n, uint32_t id_base,
                                                               const uint64_t* shortlist, int cand, int k, int kp,
                                                               int M, uint64_t* parts) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float s_red[kRerankThreads / 32];
  __shared__ float s_qscale;
  __shared__ int s_count;
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem);               // [kp]
  int8_t* q_s = reinterpret_cast<int8_t*>(smem + (size_t)kp * 8);  // [dpad]
  const int p = blockIdx.x, y = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();

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

  pdl_wait_prior();  // the shortlist is complete
  const int lane8 = lane & 7;
  const int e = p * kRerankRowsPerCta + (tid >> 3);
  const int chunks = dpad >> 4;
  int64_t local = -1;
  uint32_t gid = 0;
  if (e < cand) {
    const uint64_t key = shortlist[(size_t)y * cand + e];
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
#pragma unroll 4
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
  __syncthreads();
  const int cnt = s_count;
  for (int i = cnt + tid; i < kp; i += kRerankThreads) buf[i] = kEmptyKey;
  named_sync(1, kRerankThreads);
  group_sort_desc<kRerankThreads>(buf, kp, tid, 1);
  uint64_t* out = parts + ((size_t)p * M + y) * k;
  for (int i = tid; i < k; i += kRerankThreads) out[i] = buf[i];
}

int pow2_ceil(int x) {
  int p = 2;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace

cudaError_t binary_prep_launch(const float* q, int32_t M, int32_t d, const float* center, int32_t wpad,
                               uint64_t* qbits, unsigned int* hist, int32_t nbins, cudaStream_t stream,
                               const unsigned int* gate) {
  if (M <= 0 || d <= 0 || wpad * 64 < d) return cudaErrorInvalidValue;
  binary_prep_kernel<<<M, 1024, 0, stream>>>(q, d, center, wpad, qbits, hist, nbins, gate);
  return cudaGetLastError();
}

int32_t shortlist_segments(int32_t sm_count) { return 4 * (sm_count > 0 ? sm_count : 1); }

cudaError_t shortlist_launch(const uint16_t* dist, int64_t n, int64_t dstride, int32_t M, const unsigned int* hist,
                             int32_t nbins,
                             int32_t cand, int32_t P, unsigned int* counts, uint32_t id_base, uint64_t* out,
                             bool sorted, cudaStream_t stream, const unsigned int* gate) {
  if (M <= 0 || cand <= 0 || P <= 0 || dstride % kRowsPerThread != 0) return cudaErrorInvalidValue;
  dim3 grid((unsigned)P, (unsigned)M);
  cudaError_t e = launch_pdl(shortlist_count_kernel, grid, dim3(kSegThreads), 0, stream, dist, n, dstride, hist,
                             nbins, (int64_t)cand, P, counts, gate);
  if (e != cudaSuccess) return e;
  e = launch_pdl(shortlist_emit_kernel, grid, dim3(kSegThreads), 0, stream, dist, n, dstride, hist, nbins,
                 (int64_t)cand, P, (const unsigned int*)counts, id_base, out, gate);
  if (e != cudaSuccess || !sorted) return e;
  if (cand > kRerankMaxCand) return cudaErrorInvalidValue;
  const int candp = pow2_ceil(cand);
  e = cudaFuncSetAttribute(sort_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRerankMaxCand * 8);
  if (e != cudaSuccess) return e;
  return launch_pdl(sort_keys_kernel, dim3((unsigned)M), dim3(1024), (size_t)candp * 8, stream, out, cand, candp, gate);
}

cudaError_t sign_rows_launch(const uint64_t* bits, int64_t n, int64_t n_alloc, int32_t wpad, int32_t d, int32_t dpad,
                             int8_t* rows, cudaStream_t stream) {
  if (dpad % 16 != 0 || dpad > wpad * 64 || n > n_alloc) return cudaErrorInvalidValue;
  const int64_t threads = n_alloc * (dpad / 16);
  if (threads == 0) return cudaSuccess;
  sign_rows_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(bits, n, n_alloc, wpad, d, dpad, rows);
  return cudaGetLastError();
}

int32_t rerank_parts(int32_t cand) { return (cand + kRerankRowsPerCta - 1) / kRerankRowsPerCta; }

cudaError_t rerank_launch(const float* q, int32_t M, int32_t d, int32_t dpad, const int8_t* codes,
                          const float* scales, int64_t n, uint32_t id_base, const uint64_t* shortlist,
                          int32_t cand, int32_t k, uint64_t* parts, uint64_t* out, cudaStream_t stream) {
  if (M <= 0 || cand <= 0 || cand > kRerankMaxCand || k <= 0 || k > cand || dpad % 16 != 0)
    return cudaErrorInvalidValue;
  const int kp = pow2_ceil(k > kRerankRowsPerCta ? k : kRerankRowsPerCta);
  const int P = rerank_parts(cand);
  const size_t smem = (size_t)kp * 8 + (size_t)dpad;
  cudaError_t e = cudaFuncSetAttribute(rerank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)((size_t)kRerankMaxCand * 8 + 2048));
  if (e != cudaSuccess) return e;
  e = launch_pdl(rerank_kernel, dim3((unsigned)P, (unsigned)M), dim3(kRerankThreads), smem, stream, q, d, dpad, codes,
                 scales, n, id_base, shortlist, cand, k, kp, M, parts);
  if (e != cudaSuccess) return e;
  return merge_keys_launch(parts, P, M, k, out, stream, true);
}

}  // namespace fi8
