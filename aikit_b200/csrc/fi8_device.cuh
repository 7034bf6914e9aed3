// fi8_device.cuh -- device-side building blocks shared by the scan kernels:
// packed top-K keys, the bit-exact W8A8 query quantizer and score epilogue,
// mbarrier / bulk-copy PTX wrappers with bounded waits, and a shared-memory
// bitonic sort.
//
// Ranking key. The reference ranks hits by (score desc, index asc) with NaN
// rejected (topk/topk.go:95, topk/cmp.go:15-26, ann/flat_i8.go:233-238). A hit
// is packed into one uint64 so that a larger key is a better hit:
//   bits 63..32  order-preserving image of the float32 score (-0 == +0)
//   bits 31..1   0x7FFFFFFF - index   (lower index => larger key)
//   bit  0       1 iff the score was -0.0 (restores the exact bits on unpack)
// Keys are distinct for distinct indices, so top-K of keys is a total-order
// selection: order-independent, decomposable across tiles, CTAs and GPUs.
// Key 0 is never produced (the smallest score image is 0x007FFFFF) and marks
// an empty slot.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace fi8 {

constexpr uint64_t kEmptyKey = 0ull;

__host__ __device__ __forceinline__ uint32_t score_to_ord(float f) {
#ifdef __CUDA_ARCH__
  uint32_t b = __float_as_uint(f);
#else
  uint32_t b;
  __builtin_memcpy(&b, &f, 4);
#endif
  if (b == 0x80000000u) b = 0u;  // -0 ranks equal to +0
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__host__ __device__ __forceinline__ uint64_t make_key(float score, uint32_t idx) {
#ifdef __CUDA_ARCH__
  uint32_t negzero = (__float_as_uint(score) == 0x80000000u) ? 1u : 0u;
#else
  uint32_t b;
  __builtin_memcpy(&b, &score, 4);
  uint32_t negzero = (b == 0x80000000u) ? 1u : 0u;
#endif
  return ((uint64_t)score_to_ord(score) << 32) |
         ((uint64_t)((0x7FFFFFFFu - idx) & 0x7FFFFFFFu) << 1) | negzero;
}

__host__ __device__ __forceinline__ float key_score(uint64_t key) {
  uint32_t ord = (uint32_t)(key >> 32);
  uint32_t b = (ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord;
  if (b == 0u && (key & 1ull)) b = 0x80000000u;
#ifdef __CUDA_ARCH__
  return __uint_as_float(b);
#else
  float f;
  __builtin_memcpy(&f, &b, 4);
  return f;
#endif
}

__host__ __device__ __forceinline__ int32_t key_index(uint64_t key) {
  return (int32_t)(0x7FFFFFFFu - (uint32_t)((key >> 1) & 0x7FFFFFFFull));
}

#ifdef __CUDACC__

// ---------------------------------------------------------------------------
// W8A8 arithmetic, bit-identical to linalg (quant.go:43-71, :290-296).
// ---------------------------------------------------------------------------

// The reference's max-abs step: v<0 -> -v, keep v if v > max. NaN never wins
// a comparison, so NaNs are ignored; the combine below is associative for the
// non-NaN values that can reach it, so any reduction order gives the same max.
__device__ __forceinline__ float absmax_step(float m, float v) {
  if (v < 0.0f) v = -v;
  return (v > m) ? v : m;
}
__device__ __forceinline__ float absmax_combine(float a, float b) { return (b > a) ? b : a; }

// One code: round-half-away(v*inv) clamped to +-127; NaN -> 0 (Go's amd64
// float->int conversion yields 0 for NaN).
__device__ __forceinline__ int8_t quant_code(float v, float inv) {
  float x = roundf(__fmul_rn(v, inv));
  if (x > 127.0f) x = 127.0f;
  else if (x < -127.0f) x = -127.0f;
  if (x != x) return 0;
  return (int8_t)(int)x;
}

// An IEEE binary32 multiply with the NaN results of x86 SSE (MULSS), which is
// what the reference's Go code runs on amd64: a NaN operand propagates quieted
// (the first one if both are NaN), and an invalid operation (0 * Inf) yields the
// "real indefinite" 0xFFC00000. Finite results are plain round-to-nearest.
__device__ __forceinline__ float mul_x86(float a, float b) {
  const float r = __fmul_rn(a, b);
  if (r == r) return r;
  if (a != a) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
  if (b != b) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
  return __uint_as_float(0xFFC00000u);
}

// float32(dot) * qscale * rowscale, left to right with two rounded multiplies;
// an all-zero query (qscale == 0) scores exactly 0 (quant.go:291-294).
__device__ __forceinline__ float w8a8_score(int32_t dot, float qscale, float rowscale) {
  if (qscale == 0.0f) return 0.0f;
  return mul_x86(mul_x86(__int2float_rn(dot), qscale), rowscale);
}

// ---------------------------------------------------------------------------
// Keep filters (QueryFilter's keep(id), ann/flat_i8.go:136): a bitmap over
// global row ids, bit id%64 of word id/64; ids at or past nbits are not kept.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool keep_bit(const uint64_t* keep, int64_t nbits, uint64_t id) {
  return (int64_t)id < nbits && ((__ldg(keep + (id >> 6)) >> (id & 63)) & 1ull);
}

// The 32 keep bits of ids [start, start + 32), bit i for id start + i.
__device__ __forceinline__ uint32_t keep_bits32(const uint64_t* keep, int64_t nbits, uint64_t start) {
  if ((int64_t)start >= nbits) return 0u;
  const uint64_t w = start >> 6;
  const uint32_t sh = (uint32_t)(start & 63);
  uint64_t lo = __ldg(keep + w) >> sh;
  if (sh > 32 && (int64_t)((w + 1) << 6) < nbits) lo |= __ldg(keep + w + 1) << (64 - sh);
  uint32_t bits = (uint32_t)lo;
  const int64_t valid = nbits - (int64_t)start;
  if (valid < 32) bits &= (1u << valid) - 1u;
  return bits;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL). A kernel launched with
// launch_pdl may be scheduled before the previous kernel in its stream has
// finished: pdl_launch_dependents lets the next kernel be scheduled, and
// pdl_wait_prior (per thread) waits until the previous kernel has completed
// and its memory is visible. Without a programmatic dependency both are
// no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... Exp, typename... Act>
cudaError_t launch_pdl(void (*kernel)(Exp...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Act&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Exp>(args)...);
}

// ---------------------------------------------------------------------------
// Bounded waits. Every spin in this library gives up after kWaitLimitNs of
// wall time (globaltimer), records an error and lets the kernel unwind.
// ---------------------------------------------------------------------------
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint32_t kWaitSuspendNs = 20000;          // a sleeping test gives up after 20 us at most

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (non-tensor cp.async.bulk, global -> shared).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread may sleep until the phase
// completes (or the hint runs out) instead of returning at once, so a waiting
// warp does not spin through issue slots the working warps of its SM need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kWaitSuspendNs)
      : "memory");
  return ok != 0;
}

// As mbar_wait_bounded, sleeping between tests (see mbar_try_wait_sleep).
__device__ __forceinline__ bool mbar_wait_bounded_sleep(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait_sleep(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_sleep(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// Returns false if the phase did not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------------------
// Shared-memory bitonic sort, descending, n a power of two. All threads of the
// block must call it; it ends with a barrier.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void bitonic_sort_desc(uint64_t* buf, int n) {
  const int half = n >> 1;
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const int lo = 2 * stride * (i / stride) + (i % stride);
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t a = buf[lo], b = buf[hi];
        if ((a < b) == desc) {
          buf[lo] = b;
          buf[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

#endif  // __CUDACC__

}  // namespace fi8
