// fi8_gemm.cu -- the batched FlatI8 path on sm_100a: the W8A8 scores of a
// query batch against a corpus row range as a tcgen05 kind::i8 tensor-core
// GEMM (int32 accumulators in TMEM), with the scale epilogue and an exact
// threshold filter fused, so the Q x N score matrix never reaches HBM.
//
// Reference semantics: the batch scores of ScoreBatch / MatmulBTW8A8 with M
// queries (ann/backend.go:43, linalg/quant.go:192-298) and the per-query top-K
// of TopKBatch (gpu/anncuda/backend.go:568-667, ann/flat_i8.go:214-246).
//
// Selection runs over row ranges [0,s1), [s1,s2), ... of growing size. For
// each range the GEMM keeps, per query, every row whose packed key exceeds the
// query's threshold; then select_kernel folds those candidates into the
// query's running exact top-k and sets the next threshold to its k-th best key
// -- the k-th best of k real rows already seen, so no row that can reach the
// final top-k is ever discarded. Ranges grow by a factor F, so a range admits
// about k*F candidates per query on exchangeable data, whatever N is.
//
// gemm_kernel, one persistent CTA per SM, warp-specialized (576 threads):
//   warp 0   TMA producer: per pipeline stage, a 128x128 query tile and a
//            256x128 corpus tile (both SWIZZLE_128B, K-major) -> shared memory
//   warp 1   MMA issuer: 4 x tcgen05.mma.kind::i8 (128x256x32) per stage into
//            one of two 256-column TMEM accumulators; tcgen05.commit frees the
//            stage and, after the last K stage, hands the accumulator on
//   warps 2-17 epilogue: tcgen05.ld 32 columns at a time (warp w reads TMEM
//            lanes 32*(w%4).. = its queries, and one quarter of the 256
//            columns), a branch-free float pre-filter against the query's
//            threshold, then the exact key test and append for survivors.
// Every TMA load here is a plain single-CTA load into this CTA's shared memory.
#include <cuda.h>

#include <cfloat>

#include "fi8_device.cuh"
#include "fi8_gemm.cuh"
#include "fi8_select.cuh"

namespace fi8 {

namespace {

// Query tiles of BM = 64 or 128 queries (the MMA's M). A batch of at most 64
// queries uses M = 64: half the tensor work and half the query-tile traffic of
// padding it to 128.
// A CTA pair (PAIR, tcgen05 cta_group::2) computes a 256-query x 256-row tile:
// each CTA stages its own 128 query rows and half (128) of the corpus rows,
// and the pair's M = 256 MMA reads the corpus half of both CTAs. A CTA then
// pulls 32 KB of operands per K stage instead of 48 KB for the same MMA work.
template <int BM>
__host__ __device__ constexpr int stage_a() { return BM * kGemmBK; }  // 8 / 16 KB
template <bool PAIR>
__host__ __device__ constexpr int stage_b() { return (PAIR ? kGemmBN / 2 : kGemmBN) * kGemmBK; }  // 16 / 32 KB
template <int BM, bool PAIR = false>
__host__ __device__ constexpr int stage_bytes() { return stage_a<BM>() + stage_b<PAIR>(); }
template <bool PAIR>
__host__ __device__ constexpr int stages() { return PAIR ? 6 : 4; }  // the pair's stages are 2/3 the size
constexpr int kEpiWarps = 16;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kGemmThreads = 64 + kEpiThreads;
constexpr int kTmemCols = 512;  // two 256-column accumulators
constexpr int kStageKeys = 4;   // staged candidate keys per epilogue thread
constexpr int kChunkCols = 16;  // accumulator columns an epilogue thread loads and tests at a time
template <int BM, bool PAIR>
constexpr size_t gemm_smem() { return (size_t)stages<PAIR>() * stage_bytes<BM, PAIR>() + 1024; }  // + alignment slack

// tcgen05 instruction descriptor, kind::i8: D = s32 (c_format 2), A and B
// signed 8-bit (format 1), both K-major, N = 256 (n_dim = N>>3), M = BM
// (m_dim = M>>4; the pair's M is 256).
template <int BM>
__host__ __device__ constexpr uint32_t idesc() {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kGemmBN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major SWIZZLE_128B tile whose rows
// are 128 bytes: start address >> 4, leading byte offset 1 (unused for
// swizzled K-major), stride byte offset 1024 >> 4 (8-row swizzle atoms),
// version 1, layout type 2 (128B swizzle). The tile base is 1024-aligned.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 8-byte asynchronous global -> shared copy (no registers held while in
// flight); completion by cp_async_wait_all in the issuing thread.
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int BM>
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc<BM>()), "r"(accumulate)
      : "memory");
}

// The pair's MMA (M = 256 across the two CTAs' TMEM, issued by the even CTA):
// A rows 0-127 and corpus rows 0-127 from the even CTA's shared memory, A rows
// 128-255 and corpus rows 128-255 from the odd CTA's, at the same offsets.
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc<256>()), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// The pair's commits: to the barrier at this offset in both CTAs, or in this
// CTA only.
__device__ __forceinline__ void umma_commit_pair_both(uint64_t* bar) {
  const uint16_t mask = 3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// The shared::cluster address of this CTA's variable at `p` in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of either CTA of the cluster (cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// A tiled load whose completion is counted on an mbarrier of either CTA of
// the pair (cluster address); never multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Two IEEE round-to-nearest float32 products at once (sm_100's packed f32x2
// multiply): each lane is exactly __fmul_rn of the same operands.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)));
  return *reinterpret_cast<const float2*>(&d);
}

// max(a, b, c) in one instruction (NaN operands are ignored, as fmaxf does)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// The exact W8A8 scores of a 16-column chunk, in place of its accumulators:
// float32(dot) * qs * rs, two rounded multiplies left to right per column
// (the reference's order, linalg/quant.go:290-296), the pairs multiplied
// packed. Returns their largest, NaN skipped (a NaN never passes the filter),
// so the chunk can hold a passing score only if this max passes. The plain
// product equals the x86-semantics score whenever it is not NaN.
__device__ __forceinline__ float chunk_scores_w8a8(uint32_t (&v)[kChunkCols], float qs, const float* scl) {
  const float2 q2 = make_float2(qs, qs);
  const float4* s4 = reinterpret_cast<const float4*>(scl);
  float m = -INFINITY;
#pragma unroll
  for (int i4 = 0; i4 < kChunkCols / 4; i4++) {
    const float4 rs = s4[i4];
    const float2 a0 = mul2_rn(make_float2(__int2float_rn((int32_t)v[4 * i4]), __int2float_rn((int32_t)v[4 * i4 + 1])), q2);
    const float2 a1 =
        mul2_rn(make_float2(__int2float_rn((int32_t)v[4 * i4 + 2]), __int2float_rn((int32_t)v[4 * i4 + 3])), q2);
    const float2 s0 = mul2_rn(a0, make_float2(rs.x, rs.y));
    const float2 s1 = mul2_rn(a1, make_float2(rs.z, rs.w));
    v[4 * i4] = __float_as_uint(s0.x);
    v[4 * i4 + 1] = __float_as_uint(s0.y);
    v[4 * i4 + 2] = __float_as_uint(s1.x);
    v[4 * i4 + 3] = __float_as_uint(s1.y);
    m = max3f(m, max3f(s0.x, s0.y, s1.x), s1.y);
  }
  return m;
}

// Which query of a tile an A row holds, and which query a TMEM lane's
// accumulators belong to (-1: none).
//  * BM = 64: A rows are dense; the M = 64 accumulator puts rows 16i..16i+15
//    in lanes 32i..32i+15, so every epilogue sub-partition gets 16 queries.
//  * BM = 128: A row r is TMEM lane r. A tile with at most 64 real queries
//    places them 16 per 32-lane quarter, for the same balance; a fuller tile
//    is dense.
template <int BM>
__device__ __forceinline__ int arow_query(int r, int m_t) {
  if (BM == 128 && m_t <= 64) {
    const int l = r & 31;
    return l < 16 ? ((r >> 5) << 4) + l : -1;
  }
  return r;
}
template <int BM>
__device__ __forceinline__ int lane_query(int r, int m_t) {
  if (BM == 64 || m_t <= 64) {
    const int l = r & 31;
    return l < 16 ? ((r >> 5) << 4) + l : -1;
  }
  return r;
}
// A row of query j of a tile
template <int BM>
__device__ __forceinline__ int query_arow(int j, int m_t) {
  return (BM == 128 && m_t <= 64) ? ((j >> 4) << 5) + (j & 15) : j;
}

// Move a thread's staged candidate keys into its query's global list.
__device__ __forceinline__ void flush_staged(const GemmParams& p, int q, const uint64_t* stage, int staged) {
  if (staged == 0) return;
  unsigned int pos = atomicAdd(p.cnt + q, (unsigned int)staged);
  uint64_t* dst = p.cand + (size_t)q * p.cap;
  for (int j = 0; j < staged; j++, pos++)
    if (pos < (unsigned int)p.cap) dst[pos] = stage[j];
}

// The units of one persistent CTA: unit blockIdx.x + u*G is query tile
// unit % qtiles of row tile unit / qtiles. Stepping u adds G = dq + dr*qtiles,
// so the walk advances both with an add and a compare instead of two 64-bit
// divisions per unit.
struct UnitWalk {
  int qt, dq, qtiles;
  int64_t rt, dr;
  __device__ UnitWalk(int first, int G, int qtiles_)
      : qt(first % qtiles_), dq(G % qtiles_), qtiles(qtiles_), rt(first / qtiles_), dr(G / qtiles_) {}
  __device__ __forceinline__ void next() {
    qt += dq;
    rt += dr;
    if (qt >= qtiles) {
      qt -= qtiles;
      rt++;
    }
  }
};

// PAIR (BM = 128): launched in clusters of two CTAs. Both CTAs walk the
// same units (cluster c takes units c, c + clusters, ...) over 256-query
// tiles: CTA r of the pair holds query tile 2 * tile + r and loads corpus rows
// row0 + 128 r .. + 127 of the unit's 256. Both CTAs' loads complete on the
// even CTA's full barriers; the even CTA's MMA thread issues the pair's
// M = 256 MMAs and commits to both CTAs' barriers; both CTAs' epilogues read
// their own TMEM and release the accumulator on the even CTA's barrier. A
// cluster barrier follows the set-up and precedes the teardown, so no CTA
// signals a barrier of its peer before it exists or after it is gone.
template <int BM, bool HAM, bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  static_assert(!PAIR || BM == 128, "CTA pairs use 128-query tiles");
  constexpr int kStages = stages<PAIR>();
  constexpr int kStageA = stage_a<BM>();
  constexpr int kStageBytes = stage_bytes<BM, PAIR>();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t s_full[kStages], s_empty[kStages], s_tfull[2], s_tempty[2], s_done;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;
  __shared__ __align__(16) float s_scale[kEpiWarps][2][64];  // per epilogue warp: its columns' row scales
  __shared__ uint64_t s_stage[kEpiThreads][kStageKeys];       // per epilogue thread: staged candidates

  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // unit walkers: CTAs, or CTA pairs walking 256-query tiles
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int G = PAIR ? (int)cluster_count() : (int)gridDim.x;
  const int walker = PAIR ? (int)cluster_id() : (int)blockIdx.x;
  const int wtiles = PAIR ? p.qtiles / 2 : p.qtiles;  // query tiles of the walk
  const int64_t units = (int64_t)wtiles * p.rtiles;
  const int64_t my_units = units > walker ? (units - walker + G - 1) / G : 0;
  const bool leader = rank == 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&s_tfull[b], 1);
      mbar_init(&s_tempty[b], PAIR ? 2 * kEpiWarps : kEpiWarps);  // the pair's: both CTAs' epilogues
    }
    mbar_init(&s_done, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 1) {
    if (PAIR) {  // one warp of each CTA of the pair: the same columns in both
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync();  // both CTAs' barriers and TMEM exist before either signals the other
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  pdl_launch_dependents();
  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    // The corpus tiles depend on nothing earlier in the stream; the query tile
    // A does, on the quantize kernel, which only the first range's launch
    // follows directly. Later ranges stream while the previous select runs.
    if (lane == 0) {
      if (p.producer_waits) pdl_wait_prior();
      int64_t step = 0;
      UnitWalk w(walker, G, wtiles);
      for (int64_t u = 0; u < my_units && !s_abort; u++, w.next()) {
        const int qt = PAIR ? 2 * w.qt + (int)rank : w.qt;
        // this CTA's corpus rows: the unit's 256, or its half of them
        const int32_t row0 = (int32_t)(p.row_lo + w.rt * kGemmBN) + (PAIR ? (int32_t)rank * (kGemmBN / 2) : 0);
        for (int kc = 0; kc < p.kchunks; kc++, step++) {
          const int s = (int)(step % kStages);
          if (step >= kStages && !mbar_wait_bounded_sleep(&s_empty[s], (uint32_t)(((step / kStages) - 1) & 1))) {
            s_abort = 1;
            atomicOr(p.err, 1u);
            break;
          }
          unsigned char* st = smem + (size_t)s * kStageBytes;
          if (PAIR) {
            // both CTAs' bytes complete on the even CTA's barrier
            if (leader) mbar_arrive_expect_tx(&s_full[s], 2 * kStageBytes);
            const uint32_t full = cluster_addr(&s_full[s], 0);
            tma_load_2d_pair(st, &tmA, kc * kGemmBK, qt * BM, full);
            tma_load_2d_pair(st + kStageA, &tmB, kc * kGemmBK, row0, full);
          } else {
            mbar_arrive_expect_tx(&s_full[s], kStageBytes);
            tma_load_2d(st, &tmA, kc * kGemmBK, qt * BM, &s_full[s]);
            tma_load_2d(st + kStageA, &tmB, kc * kGemmBK, row0, &s_full[s]);
          }
        }
      }
      // let issued copies land before teardown (bounded; a no-op when drained).
      // The pair's full barriers are the even CTA's and count both CTAs' bytes;
      // the odd CTA's copies have landed once its epilogue has seen the last
      // accumulator, which follows every MMA that read them.
      if (leader)
        for (int64_t j = (step > kStages ? step - kStages : 0); j < step; j++)
          mbar_wait_bounded_sleep(&s_full[j % kStages], (uint32_t)((j / kStages) & 1));
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    // (the pair's MMAs are the even CTA's)
    if (lane == 0 && leader) {
      int64_t step = 0;
      for (int64_t u = 0; u < my_units && !s_abort; u++) {
        const int b = (int)(u & 1);
        if (u >= 2 && !mbar_wait_bounded_sleep(&s_tempty[b], (uint32_t)(((u / 2) - 1) & 1))) {
          s_abort = 1;
          atomicOr(p.err, 1u);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(b * kGemmBN);
        for (int kc = 0; kc < p.kchunks; kc++, step++) {
          const int s = (int)(step % kStages);
          if (!mbar_wait_bounded_sleep(&s_full[s], (uint32_t)((step / kStages) & 1))) {
            s_abort = 1;
            atomicOr(p.err, 1u);
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + (size_t)s * kStageBytes);
          const uint32_t b_base = a_base + kStageA;
#pragma unroll
          for (int k = 0; k < kGemmBK / 32; k++) {
            // advance K by 32 bytes inside the swizzled 128-byte rows
            const uint64_t ad = sw128_desc(a_base) + (uint64_t)(2 * k), bd = sw128_desc(b_base) + (uint64_t)(2 * k);
            if (PAIR)
              umma_i8_pair(d_tmem, ad, bd, (kc > 0 || k > 0) ? 1u : 0u);
            else
              umma_i8<BM>(d_tmem, ad, bd, (kc > 0 || k > 0) ? 1u : 0u);
          }
          if (PAIR)
            umma_commit_pair_both(&s_empty[s]);  // frees the stage in both CTAs
          else
            umma_commit(&s_empty[s]);
        }
        if (s_abort) break;
        if (PAIR)
          umma_commit_pair_both(&s_tfull[b]);  // both CTAs' accumulators are ready
        else
          umma_commit(&s_tfull[b]);
      }
      // every MMA this thread issued has completed before TMEM is released
      if (PAIR)
        umma_commit_pair_local(&s_done);
      else
        umma_commit(&s_done);
      mbar_wait_bounded_sleep(&s_done, 0);
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    // Warp w reads TMEM lanes 32*(w%4).. (its queries) and columns
    // 64*((w-2)/4).. of each 256-column accumulator. Each warp stages the 64
    // row scales of its own columns in a private shared slice and loads the
    // next unit's while it filters this one, so the epilogue warps never wait
    // for one another or for a scale load.
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int cq = ew >> 2;
    const int r = quarter * 32 + lane;  // A row / TMEM lane of this thread
    float* const my_scale = &s_scale[ew][0][0];
    if (!HAM && my_units > 0) {
      const int64_t row0 = p.row_lo + ((int64_t)walker / wtiles) * kGemmBN;
      cp_async8(my_scale + 2 * lane, p.scales + row0 + cq * 64 + 2 * lane);
    }
    cp_async_commit();
    // thresholds, counts and the candidate list come from the previous select
    pdl_wait_prior();
    // per-query state of the current query tile (constant within a launch)
    // (a lane without a query gets qs = 0 and Tscore = +inf: it never passes)
    int cur_qt = -1, q = 0;
    // Whether this lane holds a query of the current tile. With 64-query
    // tiles the M = 64 MMA writes TMEM lanes 0-15 of each sub-partition only,
    // so the other lanes read stale accumulators: their mask must be empty
    // whatever those values are (their q is not a query index).
    bool lane_valid = false;
    uint64_t* const my_stage = s_stage[ew * 32 + lane];
    int staged = 0;  // candidates held in my_stage, not yet in the global list
    float qs = 0.0f, Tscore = INFINITY;
    // Hamming mode: the filter in accumulator units -- a row passes iff its
    // dot >= hthr (always inside [-ham_dim, ham_dim + 1], so hthr - 1 - dot
    // cannot overflow)
    int32_t hthr = 0;
    unsigned long long T = ~0ull;
    // The scale and threshold of this lane's query in the next unit's tile
    // are loaded one unit ahead (the tile changes from unit to unit when G is
    // not a multiple of qtiles), so their latency overlaps this unit's work.
    float qs_next = 0.0f;
    unsigned long long T_next = ~0ull;
    auto fetch_tile_state = [&](int qt_f) {
      const int m_t = min(BM, p.M - qt_f * BM);
      const int j = lane_query<BM>(r, m_t);
      const bool valid = j >= 0 && j < m_t;
      qs_next = valid ? p.qscale[qt_f * BM + query_arow<BM>(j, m_t)] : 0.0f;
      T_next = valid ? p.thr[qt_f * BM + j] : ~0ull;
    };
    // the query tile of a walk position: the walker's own, or this CTA's
    // half of the pair's 256-query tile
    auto tile_of = [&](int wqt) { return PAIR ? 2 * wqt + (int)rank : wqt; };
    UnitWalk w(walker, G, wtiles);
    if (my_units > 0) fetch_tile_state(tile_of(w.qt));
    for (int64_t u = 0; u < my_units; u++) {
      const int qt = tile_of(w.qt);
      const int64_t row0 = p.row_lo + w.rt * kGemmBN;
      const int b = (int)(u & 1);
      if (qt != cur_qt) {
        flush_staged(p, q, my_stage, staged);  // staged keys belong to the previous tile's query
        staged = 0;
        cur_qt = qt;
        const int m_t = min(BM, p.M - qt * BM);
        const int j = lane_query<BM>(r, m_t);
        const bool valid_q = j >= 0 && j < m_t;
        lane_valid = valid_q;
        q = qt * BM + j;
        qs = qs_next;  // fetched for this tile
        T = T_next;
        // T is the k-th best key of rows below this range, and every row of
        // this range has a larger index, so a row scoring exactly T's score
        // loses the (score desc, index asc) comparison: only scores strictly
        // above pass, i.e. scores >= the next float up. With no threshold
        // yet (T == 0) every non-NaN score passes, -inf included.
        Tscore = !valid_q ? INFINITY : (T == 0ull) ? -INFINITY : nextafterf(key_score(T), INFINITY);
        // scores are the integers (dot - ham_dim) / 2: score > T's score s
        // <=> dot >= ham_dim + 2 (s + 1)
        if (HAM)
          hthr = !valid_q ? p.ham_dim + 1
                 : (T == 0ull) ? -p.ham_dim
                               : p.ham_dim + 2 * ((int32_t)key_score(T) + 1);
      }
      w.next();  // from here on, the next unit's tiles
      if (u + 1 < my_units && tile_of(w.qt) != qt) fetch_tile_state(tile_of(w.qt));
      if (s_abort) break;
      // this unit's scales (copied during the previous unit) have landed;
      // start the copy of the next unit's into the other slot
      cp_async_wait_all();
      __syncwarp();
      if (!HAM && u + 1 < my_units) {
        const int64_t nrow0 = p.row_lo + w.rt * kGemmBN;
        cp_async8(my_scale + (b ^ 1) * 64 + 2 * lane, p.scales + nrow0 + cq * 64 + 2 * lane);
      }
      cp_async_commit();
      if (!mbar_wait_bounded_sleep(&s_tfull[b], (uint32_t)((u / 2) & 1))) {
        s_abort = 1;
        atomicOr(p.err, 1u);
        break;
      }
      tc_fence_after();
      const int lim = (int)min(p.row_hi - row0, (int64_t)kGemmBN);  // valid columns of this tile (32-bit compares)
      // W8A8: the largest row scale of each 16-column chunk (lane 8c holds
      // chunk c's after the group reduction) and the lanes whose two scales
      // are not finite and >= 0 (a chunk holding one gets no bound)
      float cmax = 0.0f;
      uint32_t cbad = 0u;
      if (!HAM) {
        const float2 s2 = reinterpret_cast<const float2*>(my_scale + b * 64)[lane];
        const bool ok = s2.x >= 0.0f && s2.x <= FLT_MAX && s2.y >= 0.0f && s2.y <= FLT_MAX;
        cmax = fmaxf(s2.x, s2.y);
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, off));
        cbad = __ballot_sync(0xffffffffu, !ok);
      }
#pragma unroll 1
      for (int c = 0; c < 64 / kChunkCols; c++) {
        uint32_t v[kChunkCols];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * kGemmBN + cq * 64 + c * kChunkCols), v);
        const int col0 = cq * 64 + c * kChunkCols;
        const float* scl = my_scale + b * 64 + c * kChunkCols;
        // The chunk's test first: past the first range a chunk rarely holds a
        // row above its query's threshold, so one max over its columns -- of
        // the exact scores (W8A8) or of the dots (Hamming) -- rejects it with
        // a few instructions per column. Only a chunk that passes builds the
        // exact per-column mask below.
        int32_t mx = (int32_t)v[0];
#pragma unroll
        for (int i = 1; i < kChunkCols; i++) mx = max(mx, (int32_t)v[i]);
        // (uniform over the warp: every lane takes part in the shuffle)
        const float rs_max = HAM ? 0.0f : __shfl_sync(0xffffffffu, cmax, 8 * c);
        const bool rs_ok = ((cbad >> (8 * c)) & 0xFFu) == 0u;
        bool any;
        if (HAM) {
          any = mx >= hthr;
        } else if (qs == 0.0f) {
          any = 0.0f >= Tscore;  // an all-zero query scores exactly 0
        } else {
          // A bound on the chunk's scores from its largest dot: with qs >= 0
          // and every scale of the chunk in [0, rs_max], each score is at
          // most RN(RN(mx * qs) * rs_max) when mx > 0, and at most 0 when
          // mx <= 0 (rounding is monotone). Only a chunk whose bound passes
          // gets its exact scores (in place of v), then their max is tested;
          // a chunk with a scale outside that range goes straight to them.
          const float bnd = mx > 0 ? __fmul_rn(__fmul_rn(__int2float_rn(mx), qs), rs_max) : 0.0f;
          any = !rs_ok || bnd >= Tscore;
          if (any && lane_valid) any = chunk_scores_w8a8(v, qs, scl) >= Tscore;
        }
        if (!any || !lane_valid || col0 >= lim) continue;
        // The chunk's exact mask (a chunk reaches here when any of its 32
        // lanes' queries has a column above its threshold, so the whole warp
        // runs this part far more often than one lane would need it).
        uint32_t mask = 0;
        if (HAM) {
          // Hamming mode: A and B hold +1/-1 per sign bit (0 past dim), so
          // the dot is dim - 2h. The filter is an integer compare: the sign
          // bit of hthr - 1 - dot, shifted into the mask (one funnel shift);
          // v keeps the dots and survivors get their scores when appended.
          const int32_t tm1 = hthr - 1;
#pragma unroll
          for (int i = kChunkCols - 1; i >= 0; i--)
            mask = __funnelshift_l((uint32_t)(tm1 - (int32_t)v[i]), mask, 1);
        } else {
#pragma unroll
          for (int i = 0; i < kChunkCols; i++) mask |= (__uint_as_float(v[i]) >= Tscore ? 1u : 0u) << i;
        }
        constexpr uint32_t kAll = (1u << kChunkCols) - 1u;
        if (!HAM && qs == 0.0f) {  // an all-zero query scores exactly 0
          mask = (0.0f >= Tscore) ? kAll : 0u;
#pragma unroll
          for (int i = 0; i < kChunkCols; i++) v[i] = 0u;
        }
        if (col0 + kChunkCols > lim) mask &= (1u << (uint32_t)(lim - col0)) - 1u;
        if (p.keep && mask) mask &= keep_bits32(p.keep, p.keep_nbits, (uint64_t)p.id_base + row0 + col0) & kAll;
        if (mask) {
          // Survivors go to this thread's few shared staging slots while they
          // fit; otherwise one reservation in the query's global list takes
          // the staged keys and this chunk's. A survivor whose key does not
          // beat the threshold (possible only at T's score when T is +inf)
          // leaves an empty key, which the select skips.
          const int nm = __popc(mask);
          uint64_t* dst;
          unsigned int pos, room;
          if (staged + nm <= kStageKeys) {
            dst = my_stage;
            pos = (unsigned int)staged;
            room = kStageKeys;
            staged += nm;
          } else {
            pos = atomicAdd(p.cnt + q, (unsigned int)(staged + nm));
            dst = p.cand + (size_t)q * p.cap;
            room = (unsigned int)p.cap;
            for (int j = 0; j < staged; j++, pos++)
              if (pos < room) dst[pos] = my_stage[j];
            staged = 0;
          }
          const uint32_t id0 = p.id_base + (uint32_t)(row0 + col0);
          // survivors are sparse: visit only the 4-column groups that hold one
#pragma unroll
          for (int g = 0; g < kChunkCols / 4; g++) {
            const uint32_t nib = (mask >> (4 * g)) & 0xFu;
            if (nib) {
#pragma unroll
              for (int t = 0; t < 4; t++) {
                if ((nib >> t) & 1u) {
                  const int i = 4 * g + t;
                  const float sc = HAM ? __int2float_rn(((int32_t)v[i] - p.ham_dim) >> 1) : __uint_as_float(v[i]);
                  const uint64_t key = make_key(sc, id0 + (uint32_t)i);
                  // (Hamming survivors score above T's score, so their keys
                  // always beat T)
                  if (pos < room) dst[pos] = (HAM || key > T) ? key : kEmptyKey;
                  pos++;
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          mbar_arrive_cluster(cluster_addr(&s_tempty[b], 0));  // the pair's accumulator is the even CTA's to reuse
        else
          mbar_arrive1(&s_tempty[b]);
      }
    }
    cp_async_wait_all();  // no copy into shared memory outlives the loop
    flush_staged(p, q, my_stage, staged);
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync();  // neither CTA leaves while its peer may still signal or read it
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// One CTA per A row (Mpad rows): quantize the query placed there
// (quant.go:43-71, zero scale 0; see arow_query) or zero-fill an unused row,
// and reset that query's select state.
template <int BM>
__global__ void __launch_bounds__(256) quantize_kernel(const float* q, int M, int d, int dpad, int8_t* A,
                                                       float* qscale, unsigned long long* thr, unsigned int* cnt,
                                                       uint64_t* topk, int kp) {
  __shared__ float s_red[8];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int qt = row / BM;
  const int m_t = min(BM, M - qt * BM);
  const int j = arow_query<BM>(row % BM, m_t);
  int8_t* dst = A + (size_t)row * dpad;
  if (j < 0 || j >= m_t) {  // no query at this row
    for (int i = tid; i < dpad; i += blockDim.x) dst[i] = 0;
    if (tid == 0) qscale[row] = 0.0f;
    return;
  }
  const int qi = qt * BM + j;
  const float* src = q + (size_t)qi * d;
  float m = 0.0f;
  for (int i = tid; i < d; i += blockDim.x) m = absmax_step(m, src[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = absmax_combine(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((tid & 31) == 0) s_red[tid >> 5] = m;
  __syncthreads();
  if (tid == 0) {
    float mm = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) mm = absmax_combine(mm, s_red[w]);
    s_red[0] = mm;
  }
  __syncthreads();
  const float maxabs = s_red[0];
  if (maxabs == 0.0f) {
    for (int i = tid; i < dpad; i += blockDim.x) dst[i] = 0;
    if (tid == 0) qscale[row] = 0.0f;
  } else {
    const float sc = __fdiv_rn(maxabs, 127.0f);
    const float inv = __fdiv_rn(1.0f, sc);
    for (int i = tid; i < dpad; i += blockDim.x) dst[i] = i < d ? quant_code(src[i], inv) : (int8_t)0;
    if (tid == 0) qscale[row] = sc;
  }
  if (tid == 0) {
    thr[qi] = 0ull;
    cnt[qi] = 0u;
  }
  for (int i = tid; i < kp; i += blockDim.x) topk[(size_t)qi * kp + i] = kEmptyKey;
}

// One CTA per A row, as quantize_kernel: the query's sign row for the
// Hamming mode (the packing rule of binary_prep_kernel, as +1/-1 bytes).
template <int BM>
__global__ void __launch_bounds__(256) sign_prep_kernel(const float* q, int M, int d, int dpad, const float* center,
                                                        int8_t* A, float* qscale, unsigned long long* thr,
                                                        unsigned int* cnt, uint64_t* topk, int kp) {
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int qt = row / BM;
  const int m_t = min(BM, M - qt * BM);
  const int j = arow_query<BM>(row % BM, m_t);
  int8_t* dst = A + (size_t)row * dpad;
  if (j < 0 || j >= m_t) {  // no query at this row
    for (int i = tid; i < dpad; i += blockDim.x) dst[i] = 0;
    if (tid == 0) qscale[row] = 0.0f;
    return;
  }
  const int qi = qt * BM + j;
  const float* src = q + (size_t)qi * d;
  for (int i = tid; i < dpad; i += blockDim.x) {
    int8_t sgn = 0;
    if (i < d) {
      float x = src[i];
      if (center) x = __fsub_rn(x, center[i]);
      sgn = x >= 0.0f ? (int8_t)1 : (int8_t)-1;  // NaN compares false: -1
    }
    dst[i] = sgn;
  }
  if (tid == 0) {
    qscale[row] = 1.0f;
    thr[qi] = 0ull;
    cnt[qi] = 0u;
  }
  for (int i = tid; i < kp; i += blockDim.x) topk[(size_t)qi * kp + i] = kEmptyKey;
}

// One CTA per query (1024 or 512 threads): fold this range's candidates into the
// running top-k. The carried list holds keys of earlier ranges (all above the
// threshold the candidates passed), so top-k of the union is exact.
//
// An MSD radix select (8-bit digits, most significant first) over the union,
// read from global memory (L2) on every pass, finds the digit prefix that
// exactly the k best keys match or exceed: keys are distinct, so the walk ends
// at a digit bucket whose whole count is still needed. One more pass keeps
// those keys. Shared memory holds only the histogram and the kept list, so
// many queries' CTAs share an SM and a large batch selects in one wave. Only
// the last range's select orders its keys (its output is the answer).
// Threads and unrolled loads per CTA: a one-wave launch stages its union in
// shared memory (one CTA per SM) and spreads it over 1024 threads; a larger
// batch streams unions from L2 with eight 256-thread CTAs per SM (at least
// 256 threads: one per radix bin). A union there is a few thousand keys, so
// its passes are short and the launch's waves dominate: 256 threads x 4
// loads halved the selects of a 4096-query batch against 512 x 8 (0.40 ms
// against 0.79-0.83 per batch over 6.25M rows).
constexpr int kSelThreadsStaged = 1024, kSelUnrollStaged = 4;
constexpr int kSelThreads = 256, kSelUnroll = 4;
constexpr int kRadixBins = 256;
static_assert(kSelThreads >= kRadixBins && kSelThreadsStaged >= kRadixBins,
              "the select clears its histogram with one thread per radix bin");

// Slot i of a query's union: its carried list, then this range's candidates.
__device__ __forceinline__ uint64_t union_key(const uint64_t* mine, int kp, const uint64_t* src, int n_all, int i) {
  if (i >= n_all) return kEmptyKey;
  return i < kp ? __ldcg(mine + i) : __ldcg(src + (i - kp));
}

template <int NT, int UNROLL>
__global__ void __launch_bounds__(NT)
    select_kernel(int k, int kp, int cap_s, uint64_t* topk, unsigned long long* thr, unsigned int* cnt,
                  const uint64_t* cand, int cap, uint64_t* out, unsigned int* err) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_count;
  __shared__ unsigned long long s_prefix, s_mask, s_min, s_and, s_or;
  __shared__ unsigned int s_hist[kRadixBins];
  __shared__ int s_rank, s_done;
  uint64_t* sel = reinterpret_cast<uint64_t*>(smem);  // [kp] the kept keys
  uint64_t* ranked = sel + kp;                          // [kp] their order (last range)
  uint64_t* ubuf = ranked + kp;                         // [cap_s] the union, when staged
  const int qi = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  // The next range's GEMM may start early only when this select is one wave
  // (a CTA per query, at most one per SM: the staged form): its persistent
  // CTAs then take the SMs the select leaves idle and stream their first
  // corpus tiles meanwhile. A select of several waves releases it as its CTAs
  // exit: an early GEMM would take the SMs its later waves need, and while it
  // waits for their thresholds it burns power the capped clock pays for (a
  // full C3 step, batch 4096: 175 ms with the early start, 157 without).
  if (cap_s > 0) pdl_launch_dependents();
  pdl_wait_prior();  // the range's GEMM has completed
  uint64_t* mine = topk + (size_t)qi * kp;
  const unsigned int c_all = cnt[qi];
  if (c_all > (unsigned int)cap && tid == 0) atomicOr(err, 2u);  // candidates were dropped
  const int n_c = (int)(c_all < (unsigned int)cap ? c_all : (unsigned int)cap);
  const uint64_t* src = cand + (size_t)qi * cap;
  const int n_all = kp + n_c;  // slots of the union; empty keys (0) are skipped
  // A union that fits the shared buffer (one CTA per query in a single wave
  // can afford a large one) is read from L2 once; otherwise every pass reads
  // it from L2.
  const bool staged = n_all <= cap_s;
  if (staged) {
    for (int i0 = 0; i0 < n_all; i0 += NT * UNROLL) {
      uint64_t keys[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; u++) keys[u] = union_key(mine, kp, src, n_all, i0 + u * NT + tid);
#pragma unroll
      for (int u = 0; u < UNROLL; u++)
        if (i0 + u * NT + tid < n_all) ubuf[i0 + u * NT + tid] = keys[u];
    }
  }
  auto key_at = [&](int i) -> uint64_t {
    if (staged) return i < n_all ? ubuf[i] : kEmptyKey;
    return union_key(mine, kp, src, n_all, i);
  };
  if (tid == 0) {
    s_prefix = 0ull;
    s_mask = 0ull;
    s_min = ~0ull;
    s_and = ~0ull;
    s_or = 0ull;
    s_rank = k;
    s_done = 0;
    s_count = 0;
  }
  __syncthreads();
  // The first pass also ANDs and ORs every key: a later digit that all keys
  // share is appended to the prefix without a pass (score images and row ids
  // leave several bytes constant across a union).
  for (int shift = 56; shift >= 0; shift -= 8) {
    if (shift < 56 && (unsigned int)((s_and ^ s_or) >> shift & 0xFFull) == 0u) {
      __syncthreads();  // every thread has read s_and / s_or
      if (tid == 0) {
        s_prefix |= s_and & (0xFFull << shift);
        s_mask |= 0xFFull << shift;
      }
      __syncthreads();
      continue;
    }
    if (tid < kRadixBins) s_hist[tid] = 0u;
    __syncthreads();
    const unsigned long long prefix = s_prefix, mask = s_mask;
    unsigned long long k_and = ~0ull, k_or = 0ull;
    for (int i0 = 0; i0 < n_all; i0 += NT * UNROLL) {
      uint64_t keys[UNROLL];  // loads first, so their L2 latencies overlap
#pragma unroll
      for (int u = 0; u < UNROLL; u++) keys[u] = key_at(i0 + u * NT + tid);
#pragma unroll
      for (int u = 0; u < UNROLL; u++) {
        const uint64_t key = keys[u];
        const bool live = key != kEmptyKey && (key & mask) == prefix;
        const unsigned int bin = live ? (unsigned int)(key >> shift) & 0xFFu : 0x100u;
        const unsigned int same = __match_any_sync(0xffffffffu, bin);
        if (live && lane == __ffs(same) - 1) atomicAdd(&s_hist[bin], (unsigned int)__popc(same));
        if (shift == 56 && live) {
          k_and &= key;
          k_or |= key;
        }
      }
    }
    if (shift == 56) {
      const unsigned int a_lo = __reduce_and_sync(0xffffffffu, (unsigned int)k_and);
      const unsigned int a_hi = __reduce_and_sync(0xffffffffu, (unsigned int)(k_and >> 32));
      const unsigned int o_lo = __reduce_or_sync(0xffffffffu, (unsigned int)k_or);
      const unsigned int o_hi = __reduce_or_sync(0xffffffffu, (unsigned int)(k_or >> 32));
      if (lane == 0) {
        atomicAnd(&s_and, ((unsigned long long)a_hi << 32) | a_lo);
        atomicOr(&s_or, ((unsigned long long)o_hi << 32) | o_lo);
      }
    }
    __syncthreads();
    if (tid < 32) {
      // lane l holds bins 255-8l .. 248-8l (descending); find the bin where
      // the running count from the top reaches the rank
      unsigned int c[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        c[j] = s_hist[255 - 8 * lane - j];
        sum += c[j];
      }
      unsigned int incl = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const unsigned int t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
      }
      const unsigned int total = __shfl_sync(0xffffffffu, incl, 31);
      const unsigned int rank = (unsigned int)s_rank;
      if (shift == 56 && total <= rank) {
        if (lane == 0) s_done = 2;  // k or fewer keys in all: keep them all
      } else {
        const unsigned int excl = incl - sum;
        const unsigned int hit = __ballot_sync(0xffffffffu, excl < rank && rank <= incl);
        if (lane == __ffs(hit) - 1) {
          unsigned int cum = excl;
#pragma unroll
          for (int j = 0; j < 8; j++) {
            if (cum + c[j] >= rank) {
              const unsigned int digit = 255u - 8u * lane - j;
              s_prefix = prefix | ((unsigned long long)digit << shift);
              s_mask = mask | (0xFFull << shift);
              s_rank = (int)(rank - cum);
              s_done = (c[j] == rank - cum) ? 1 : 0;
              break;
            }
            cum += c[j];
          }
        }
      }
    }
    __syncthreads();
    if (s_done) break;
  }
  // keep every non-empty key at or above the prefix (exactly min(total, k))
  const unsigned long long prefix = s_done == 2 ? 0ull : s_prefix;
  const unsigned long long mask = s_done == 2 ? 0ull : s_mask;
  unsigned long long my_min = ~0ull;
  for (int i0 = 0; i0 < n_all; i0 += NT * UNROLL) {
    uint64_t keys[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; u++) keys[u] = key_at(i0 + u * NT + tid);
#pragma unroll
    for (int u = 0; u < UNROLL; u++) {
      const uint64_t key = keys[u];
      const bool take = key != kEmptyKey && (key & mask) >= prefix;
      if (take && key < my_min) my_min = key;
      warp_append(take, key, sel, &s_count);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, my_min, off);
    if (o < my_min) my_min = o;
  }
  if (lane == 0 && my_min != ~0ull) atomicMin(&s_min, my_min);
  __syncthreads();
  const int nkept = s_count;
  const uint64_t* kept = sel;
  if (out) {
    if (nkept <= 512) {
      // rank placement: a kept key's position is the number of kept keys
      // above it (keys are distinct); a sorting network beyond that
      for (int i = tid; i < nkept; i += NT) {
        const uint64_t key = sel[i];
        int rank = 0;
        for (int j = 0; j < nkept; j++) rank += sel[j] > key;
        ranked[rank] = key;
      }
    } else {
      for (int i = tid; i < kp; i += NT) ranked[i] = i < nkept ? sel[i] : kEmptyKey;
      named_sync(1, NT);
      group_sort_desc<NT>(ranked, kp, tid, 1);
    }
    __syncthreads();
    kept = ranked;
  }
  for (int i = tid; i < kp; i += NT) mine[i] = i < nkept ? kept[i] : kEmptyKey;
  if (out)
    for (int i = tid; i < k; i += NT) out[(size_t)qi * k + i] = i < nkept ? kept[i] : kEmptyKey;
  if (tid == 0) {
    thr[qi] = nkept >= k ? s_min : 0ull;
    cnt[qi] = 0u;
  }
}

// One thread, after a batch's last select: move the dropped-candidate flag
// (bit 1 of the error word) into the redo gate and clear it there, so the
// gated redo that follows runs exactly when this batch needs it and the
// flag never outlives its batch.
__global__ void overflow_latch_kernel(unsigned int* err, unsigned int* gate) {
  pdl_launch_dependents();
  pdl_wait_prior();  // the batch's selects have completed
  const unsigned int v = atomicAnd(err, ~2u);
  *gate = (v >> 1) & 1u;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// Tensor-pipe probe: back-to-back tcgen05.mma.kind::i8 (M=128, N=256, K=32)
// on operands resident in shared memory (filled with a hash pattern, so the
// multipliers toggle as on real data), accumulating into TMEM: no global
// traffic, one issuing thread per SM. Each instruction is 2*128*256*32 ops.
__global__ void __launch_bounds__(128, 1) mma_probe_kernel(int64_t iters, unsigned int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t s_done;
  __shared__ uint32_t s_tmem;
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x;
  constexpr int kBytes = stage_bytes<128>();
  for (int i = tid; i < kBytes / 4; i += blockDim.x) {
    uint32_t h = (uint32_t)i * 0x9E3779B1u + blockIdx.x;
    h ^= h >> 15;
    h *= 0x85EBCA77u;
    reinterpret_cast<uint32_t*>(smem)[i] = h ^ (h >> 13);
  }
  if (tid == 0) {
    mbar_init(&s_done, 1);
    fence_mbar_init();
  }
  if (tid < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // the operands were written by ordinary stores; the tensor core reads them
  // through the async proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  if (tid == 0) {
    const uint32_t a_base = smem_u32(smem);
    const uint32_t b_base = a_base + stage_a<128>();
    for (int64_t i = 0; i < iters; i++) {
#pragma unroll
      for (int k = 0; k < kGemmBK / 32; k++)
        umma_i8<128>(tmem, sw128_desc(a_base) + (uint64_t)(2 * k), sw128_desc(b_base) + (uint64_t)(2 * k),
                     (i > 0 || k > 0) ? 1u : 0u);
    }
    umma_commit(&s_done);
    if (!mbar_wait_bounded(&s_done, 0)) atomicOr(err, 1u);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid < 32) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
}

}  // namespace

cudaError_t mma_probe_launch(int32_t G, int64_t iters, unsigned int* err, cudaStream_t stream) {
  const size_t smem = (size_t)stage_bytes<128>() + 1024;
  cudaError_t e = cudaFuncSetAttribute(mma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  mma_probe_kernel<<<G, 128, smem, stream>>>(iters, err);
  return cudaGetLastError();
}

double mma_probe_ops(int32_t G, int64_t iters) { return 2.0 * 128 * 256 * kGemmBK * (double)iters * G; }

cudaError_t overflow_latch_launch(unsigned int* err, unsigned int* gate, cudaStream_t stream) {
  return launch_pdl(overflow_latch_kernel, dim3(1), dim3(1), 0, stream, err, gate);
}

int32_t select_max_k() { return 4096; }  // kp <= 4096 keeps the select buffer at 64 KB

bool make_tmap_i8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t pitch, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || pitch % 16 != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  const cuuint64_t dims[2] = {pitch, rows};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {(cuuint32_t)kGemmBK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BM, bool HAM, bool PAIR>
static cudaError_t gemm_launch_t(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p, int32_t G,
                                 cudaStream_t stream) {
  auto kern = gemm_kernel<BM, HAM, PAIR>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<BM, PAIR>());
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = PAIR ? 2 : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = gemm_smem<BM, PAIR>();
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = PAIR ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, p);
}

cudaError_t gemm_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p, int32_t G, int32_t bm,
                        bool pair, cudaStream_t stream) {
  const bool ham = p.ham_dim > 0;
  if (pair) {
    if (bm != 128 || G % 2 != 0 || p.qtiles % 2 != 0) return cudaErrorInvalidValue;
    return ham ? gemm_launch_t<128, true, true>(tmA, tmB, p, G, stream)
               : gemm_launch_t<128, false, true>(tmA, tmB, p, G, stream);
  }
  if (bm == 64)
    return ham ? gemm_launch_t<64, true, false>(tmA, tmB, p, G, stream)
               : gemm_launch_t<64, false, false>(tmA, tmB, p, G, stream);
  if (bm != 128) return cudaErrorInvalidValue;
  return ham ? gemm_launch_t<128, true, false>(tmA, tmB, p, G, stream)
             : gemm_launch_t<128, false, false>(tmA, tmB, p, G, stream);
}

int32_t gemm_pair_max_clusters() {
  static int32_t n = [] {
    auto kern = gemm_kernel<128, false, true>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<128, true>()) !=
        cudaSuccess)
      return 0;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = gemm_smem<128, true>();
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, kern, &cfg) != cudaSuccess) return 0;
    return (int32_t)c;
  }();
  return n;
}

cudaError_t quantize_launch(const float* q, int32_t M, int32_t Mpad, int32_t d, int32_t dpad, int8_t* A,
                            float* qscale, unsigned long long* thr, unsigned int* cnt, uint64_t* topk, int32_t kp,
                            int32_t bm, cudaStream_t stream) {
  if (bm == 64)
    quantize_kernel<64><<<Mpad, 256, 0, stream>>>(q, M, d, dpad, A, qscale, thr, cnt, topk, kp);
  else
    quantize_kernel<128><<<Mpad, 256, 0, stream>>>(q, M, d, dpad, A, qscale, thr, cnt, topk, kp);
  return cudaGetLastError();
}

cudaError_t sign_prep_launch(const float* q, int32_t M, int32_t Mpad, int32_t d, int32_t dpad, const float* center,
                             int8_t* A, float* qscale, unsigned long long* thr, unsigned int* cnt, uint64_t* topk,
                             int32_t kp, int32_t bm, cudaStream_t stream) {
  if (bm == 64)
    sign_prep_kernel<64><<<Mpad, 256, 0, stream>>>(q, M, d, dpad, center, A, qscale, thr, cnt, topk, kp);
  else
    sign_prep_kernel<128><<<Mpad, 256, 0, stream>>>(q, M, d, dpad, center, A, qscale, thr, cnt, topk, kp);
  return cudaGetLastError();
}

cudaError_t select_launch(int32_t M, int32_t k, int32_t kp, uint64_t* topk, unsigned long long* thr,
                          unsigned int* cnt, const uint64_t* cand, int32_t cap, uint64_t* out, unsigned int* err,
                          int32_t sm_count, cudaStream_t stream) {
  if (kp > 4096 || kp < k) return cudaErrorInvalidValue;
  // one wave of CTAs (a query each) stages its union in shared memory
  const int cap_s = M <= sm_count ? 16384 : 0;
  const size_t smem = (size_t)(2 * kp + cap_s) * 8;  // kept list + its order (+ the union)
  auto kern = cap_s ? select_kernel<kSelThreadsStaged, kSelUnrollStaged> : select_kernel<kSelThreads, kSelUnroll>;
  const int nt = cap_s ? kSelThreadsStaged : kSelThreads;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (2 * 4096 + 16384) * 8);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3((unsigned)M), dim3(nt), smem, stream, k, kp, cap_s, topk, thr, cnt, cand, cap, out, err);
}

}  // namespace fi8
