// fi8_scan.cu -- the batch-1 FlatI8 scan on sm_100a: an HBM-streaming int8
// GEMV with the W8A8 epilogue and an exact fused top-K.
//
// Reference semantics: w8a8Span (linalg/quant.go:248-298) for the scores,
// topHits (ann/flat_i8.go:214-246) for the selection, and the device kernels it
// replaces, gemv_w8a8 + topk_rows/topk_split/topk_merge
// (gpu/anncuda/gemv_w8a8.cu:76-130, :480-669).
//
// Structure (one CTA per SM, persistent over row tiles):
//   * thread 0 streams R-row tiles of the corpus (R*dpad contiguous bytes plus
//     R scales) into a STAGES-deep shared-memory ring with cp.async.bulk,
//     completion tracked by one mbarrier per stage;
//   * every CTA quantizes its query in shared memory (bit-identical to
//     quantizeRowInt8), then 8 lanes per row dot 16-byte chunks with dp4a and
//     reduce with warp shuffles;
//   * top-K: candidates above the CTA threshold go to a shared-memory buffer;
//     when it fills, a bitonic sort keeps the best k and raises the threshold,
//     which is also published to a per-query global threshold (atomicMax) that
//     every CTA reads back each tile. The threshold is always the k-th best key
//     of k real rows, so nothing that can reach the global top-k is dropped;
//   * the last CTA to finish (ticket counter) merges the per-CTA survivors and
//     writes the final sorted keys, then resets the per-query scratch.
#include "fi8_device.cuh"
#include "fi8_scan.cuh"

namespace fi8 {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowsPerPass = kWarps * 4;  // 8 lanes per row, 4 rows per warp
constexpr size_t kSmemBudget = 220 * 1024;

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ int next_pow2(int x) {
  int p = 2;
  while (p < x) p <<= 1;
  return p;
}

// Append `key` (when take) to buf using one shared atomic per warp.
__device__ __forceinline__ void warp_append(bool take, uint64_t key, uint64_t* buf, int* s_count) {
  const uint32_t mask = __ballot_sync(0xffffffffu, take);
  if (mask == 0) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(mask) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(s_count, __popc(mask));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (take) buf[base + __popc(mask & lanemask_lt())] = key;
}

// Sort the first cnt entries of buf, keep the best k, raise the CTA threshold
// and optionally publish it. Uniform: all threads call with the same cnt.
__device__ void compact(uint64_t* buf, int cnt, int k, int* s_count, unsigned long long* s_local_thr,
                        unsigned long long* gthr) {
  const int n2 = next_pow2(cnt < 2 ? 2 : cnt);
  for (int i = cnt + threadIdx.x; i < n2; i += blockDim.x) buf[i] = kEmptyKey;
  __syncthreads();
  bitonic_sort_desc(buf, n2);
  if (threadIdx.x == 0) {
    *s_count = cnt < k ? cnt : k;
    if (cnt >= k) {
      const unsigned long long t = buf[k - 1];
      if (t > *s_local_thr) *s_local_thr = t;
      if (gthr) atomicMax(gthr, t);
    }
  }
  __syncthreads();
}

template <bool TOPK>
__global__ void __launch_bounds__(kThreads, 1) scan_kernel(ScanParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float s_red[kWarps];
  __shared__ float s_qscale;
  __shared__ int s_count;
  __shared__ int s_abort;
  __shared__ int s_last;
  __shared__ unsigned long long s_thr;
  __shared__ unsigned long long s_local_thr;
  __shared__ int s_off[1025];

  const int G = gridDim.x;
  const int cta = blockIdx.x;
  const int y = blockIdx.y;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int R = p.rows_per_tile;
  const int dpad = p.dpad;
  const int S = p.stages;
  const uint32_t code_bytes = (uint32_t)R * (uint32_t)dpad;
  const uint32_t stage_bytes = code_bytes + (uint32_t)R * 4u;

  unsigned char* stages = smem;
  int8_t* q_s = reinterpret_cast<int8_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes + (size_t)dpad);
  uint64_t* bars = buf + (TOPK ? p.cap : 0);

  const int64_t my_tiles = (p.ntiles > cta) ? (p.ntiles - cta + G - 1) / G : 0;

  if (tid == 0) {
    for (int s = 0; s < S; s++) mbar_init(&bars[s], 1);
    fence_mbar_init();
    s_count = 0;
    s_abort = 0;
    s_local_thr = 0;
    s_thr = TOPK ? ld_relaxed_u64(p.gthr + y) : 0ull;
  }
  __syncthreads();

  auto issue = [&](int64_t it) {
    const int s = (int)(it % S);
    const int64_t tile = cta + it * G;
    unsigned char* st = stages + (size_t)s * stage_bytes;
    mbar_arrive_expect_tx(&bars[s], stage_bytes);
    bulk_g2s(st, p.codes + (size_t)tile * code_bytes, code_bytes, &bars[s]);
    bulk_g2s(st + code_bytes, p.scales + (size_t)tile * R, (uint32_t)R * 4u, &bars[s]);
  };
  if (tid == 0) {
    const int64_t pre = my_tiles < S ? my_tiles : S;
    for (int64_t it = 0; it < pre; it++) issue(it);
  }

  // ---- quantize this CTA's query into shared memory (quant.go:43-71) ----
  const float* q = p.q + (size_t)y * p.d;
  float m = 0.0f;
  for (int i = tid; i < p.d; i += kThreads) m = absmax_step(m, q[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = absmax_combine(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) s_red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < kWarps ? s_red[lane] : 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = absmax_combine(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) s_red[0] = m;
  }
  __syncthreads();
  const float maxabs = s_red[0];
  if (maxabs == 0.0f) {
    for (int i = tid; i < dpad; i += kThreads) q_s[i] = 0;
    if (tid == 0) s_qscale = 0.0f;
  } else {
    const float sc = __fdiv_rn(maxabs, 127.0f);
    const float inv = __fdiv_rn(1.0f, sc);
    for (int i = tid; i < dpad; i += kThreads) q_s[i] = i < p.d ? quant_code(q[i], inv) : (int8_t)0;
    if (tid == 0) s_qscale = sc;
  }
  __syncthreads();
  const float qscale = s_qscale;

  // ---- main loop over this CTA's tiles ----
  const int chunks = dpad >> 4;
  const int lane8 = lane & 7;
  int64_t it = 0;
  for (; it < my_tiles; it++) {
    const int s = (int)(it % S);
    const uint32_t par = (uint32_t)((it / S) & 1);
    if (!mbar_wait_bounded(&bars[s], par)) {
      s_abort = 1;
      atomicOr(p.err, 1u);
    }
    const int64_t row0 = (cta + it * G) * (int64_t)R;
    const unsigned char* st = stages + (size_t)s * stage_bytes;
    const float* sc_s = reinterpret_cast<const float*>(st + code_bytes);
    const unsigned long long thr = TOPK ? s_thr : 0ull;
    for (int pass = 0; pass < R; pass += kRowsPerPass) {
      const int r = pass + warp * 4 + (lane >> 3);
      const int4* rowp = reinterpret_cast<const int4*>(st + (size_t)r * dpad);
      const int4* qp = reinterpret_cast<const int4*>(q_s);
      int acc = 0;
#pragma unroll 4
      for (int c = lane8; c < chunks; c += 8) {
        const int4 a = rowp[c];
        const int4 b = qp[c];
        acc = __dp4a(a.x, b.x, acc);
        acc = __dp4a(a.y, b.y, acc);
        acc = __dp4a(a.z, b.z, acc);
        acc = __dp4a(a.w, b.w, acc);
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      const int64_t g = row0 + r;
      const bool mine = (lane8 == 0) && (g < p.n);
      float score = 0.0f;
      if (mine) score = w8a8_score(acc, qscale, sc_s[r]);
      if (TOPK) {
        uint64_t key = kEmptyKey;
        bool take = false;
        if (mine && score == score) {
          key = make_key(score, p.id_base + (uint32_t)g);
          take = key > thr;
        }
        warp_append(take, key, buf, &s_count);
      } else {
        if (mine) p.out_scores[(size_t)y * p.n + g] = score;
      }
    }
    __syncthreads();
    if (s_abort) break;
    if (tid == 0 && it + S < my_tiles) issue(it + S);
    if (TOPK) {
      const int cnt = s_count;
      if (cnt > p.cap - R) compact(buf, cnt, p.k, &s_count, &s_local_thr, p.gthr + y);
      if (tid == 0) {
        const unsigned long long gt = ld_relaxed_u64(p.gthr + y);
        s_thr = gt > s_local_thr ? gt : s_local_thr;
      }
      __syncthreads();
    }
  }

  if (s_abort) {
    // Let the copies this CTA started land before it exits (bounded).
    if (tid == 0) {
      const int64_t last = (it + S < my_tiles) ? it + S : my_tiles;
      for (int64_t j = it; j < last; j++) mbar_wait_bounded(&bars[j % S], (uint32_t)((j / S) & 1));
    }
    __syncthreads();
  }

  if (!TOPK) return;

  // ---- per-CTA result: best k, filtered by the current shared threshold ----
  {
    const int cnt = s_abort ? 0 : s_count;
    compact(buf, cnt, p.k, &s_count, &s_local_thr, p.gthr + y);
  }
  if (tid == 0) s_thr = ld_relaxed_u64(p.gthr + y);
  __syncthreads();
  const int have = s_count;
  const unsigned long long T = s_thr;
  uint64_t* my_part = p.part_keys + ((size_t)y * G + cta) * p.k;
  // buf[0..have) is sorted descending; keep the prefix with key >= T.
  int keep = 0;
  {
    // count via ballot over the sorted prefix
    for (int base = 0; base < have; base += kThreads) {
      const int i = base + tid;
      const int ok = (i < have && buf[i] >= T) ? 1 : 0;
      const int c = __syncthreads_count(ok);
      keep += c;
      if (c < kThreads) break;
    }
  }
  for (int i = tid; i < keep; i += kThreads) my_part[i] = buf[i];
  if (tid == 0) p.part_counts[(size_t)y * G + cta] = keep;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int ticket = atomicAdd(p.counter + y, 1u);
    s_last = (ticket == (unsigned int)(G - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (!s_last) return;

  // ---- last CTA: merge the G survivor lists for query y ----
  __threadfence();
  if (tid == 0) {
    s_thr = ld_relaxed_u64(p.gthr + y);
    s_count = 0;
    s_local_thr = 0;
  }
  // exclusive prefix of the G counts (warp 0, 32 at a time)
  if (warp == 0) {
    int run = 0;
    for (int b = 0; b < G; b += 32) {
      const int i = b + lane;
      int v = (i < G) ? __ldcg(p.part_counts + (size_t)y * G + i) : 0;
      int x = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += t;
      }
      if (i < G) s_off[i] = run + x - v;
      run += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) s_off[G] = run;
  }
  __syncthreads();
  const int total = s_off[G];
  const unsigned long long Tf = s_thr;
  for (int base = 0; base < total; base += kThreads) {
    const int e = base + tid;
    bool take = false;
    uint64_t key = kEmptyKey;
    if (e < total) {
      int lo = 0, hi = G;  // find l with s_off[l] <= e < s_off[l+1]
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_off[mid] <= e) lo = mid;
        else hi = mid;
      }
      key = __ldcg(p.part_keys + ((size_t)y * G + lo) * p.k + (e - s_off[lo]));
      take = key >= Tf && key > s_local_thr;
    }
    warp_append(take, key, buf, &s_count);
    __syncthreads();
    const int cnt = s_count;
    if (cnt > p.cap - kThreads) compact(buf, cnt, p.k, &s_count, &s_local_thr, nullptr);
  }
  compact(buf, s_count, p.k, &s_count, &s_local_thr, nullptr);
  const int fin = s_count;
  for (int i = tid; i < p.k; i += kThreads) p.out_keys[(size_t)y * p.k + i] = i < fin ? buf[i] : kEmptyKey;
  if (tid == 0) {
    p.counter[y] = 0u;
    p.gthr[y] = 0ull;
  }
}

// ---------------------------------------------------------------------------
// merge_keys_kernel: top-k of nsrc candidate lists per query, one CTA each.
// Used for the cross-GPU merge after the all-gather (the 8-way analogue of
// queryBatchSharded's merge, ann/backend.go:262-277).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
    merge_keys_kernel(const uint64_t* in, int nsrc, int M, int k, int cap, uint64_t* out) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_count;
  __shared__ unsigned long long s_local_thr;
  uint64_t* buf = reinterpret_cast<uint64_t*>(smem);
  const int y = blockIdx.x;
  if (threadIdx.x == 0) {
    s_count = 0;
    s_local_thr = 0;
  }
  __syncthreads();
  const int total = nsrc * k;
  for (int base = 0; base < total; base += kThreads) {
    const int e = base + threadIdx.x;
    bool take = false;
    uint64_t key = kEmptyKey;
    if (e < total) {
      const int src = e / k, j = e - src * k;
      key = in[((size_t)src * M + y) * k + j];
      take = key != kEmptyKey && key > s_local_thr;
    }
    warp_append(take, key, buf, &s_count);
    __syncthreads();
    const int cnt = s_count;
    if (cnt > cap - kThreads) compact(buf, cnt, k, &s_count, &s_local_thr, nullptr);
  }
  compact(buf, s_count, k, &s_count, &s_local_thr, nullptr);
  const int fin = s_count;
  for (int i = threadIdx.x; i < k; i += kThreads) out[(size_t)y * k + i] = i < fin ? buf[i] : kEmptyKey;
}

int pow2_at_least(int x) {
  int p = 2;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace

bool scan_geometry(int32_t dpad, int32_t k, bool topk, ScanGeometry* g) {
  if (dpad <= 0 || dpad % 16 != 0 || dpad > kScanMaxDpad) return false;
  // Rows per tile: a power-of-two multiple of 32 (so it divides the 256-row
  // allocation padding) with a tile of at most 48 KB of codes.
  int R = 32;
  while (R < 256 && (size_t)(2 * R) * dpad <= 48 * 1024) R *= 2;
  const size_t stage = (size_t)R * (dpad + 4);
  int cap = 0;
  if (topk) {
    if (k <= 0) return false;
    // Room for k survivors plus one full tile (scan) or one 256-key chunk
    // (merge) of new candidates between compactions.
    cap = pow2_at_least(k + 256);
    if (cap > kScanMaxCap) return false;
  }
  const size_t fixed = (size_t)dpad + (size_t)cap * 8 + 64;
  int stages = 4;
  while (stages > 2 && fixed + stages * stage > kSmemBudget) stages--;
  if (fixed + stages * stage > kSmemBudget) return false;
  g->rows_per_tile = R;
  g->stages = stages;
  g->cap = cap;
  g->smem_bytes = fixed + stages * stage;
  return true;
}

cudaError_t scan_launch(const ScanParams& p, bool topk, int32_t M, int32_t G, size_t smem,
                        cudaStream_t stream) {
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(scan_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSmemBudget);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(scan_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemBudget);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(merge_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemBudget);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  if (G > 1024) return cudaErrorInvalidValue;
  dim3 grid((unsigned)G, (unsigned)M);
  if (topk)
    scan_kernel<true><<<grid, kThreads, smem, stream>>>(p);
  else
    scan_kernel<false><<<grid, kThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t merge_keys_launch(const uint64_t* in, int32_t nsrc, int32_t M, int32_t k, uint64_t* out,
                              cudaStream_t stream) {
  if (k <= 0 || k > kMergeMaxK || nsrc <= 0 || M <= 0) return cudaErrorInvalidValue;
  const int cap = pow2_at_least(k + kThreads);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(merge_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSmemBudget);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  merge_keys_kernel<<<M, kThreads, (size_t)cap * 8, stream>>>(in, nsrc, M, k, cap, out);
  return cudaGetLastError();
}

}  // namespace fi8
