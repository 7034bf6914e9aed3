// fi8_scan.cu -- the batch-1 FlatI8 scan on sm_100a: an HBM-streaming int8
// GEMV with the W8A8 epilogue and an exact fused top-K.
//
// Reference semantics: w8a8Span (linalg/quant.go:248-298) for the scores,
// topHits (ann/flat_i8.go:214-246) for the selection, and the device kernels it
// replaces, gemv_w8a8 + topk_rows/topk_split/topk_merge
// (gpu/anncuda/gemv_w8a8.cu:76-130, :480-669).
//
// One persistent CTA per SM, warp-specialized:
//   * warp 16 (producer): streams R-row tiles of the corpus (R*dpad contiguous
//     bytes plus R scales) into an S-deep shared-memory ring with
//     cp.async.bulk; a "full" mbarrier per stage counts the bytes, an "empty"
//     mbarrier per stage counts the consumer warps that are done with it;
//   * warps 0-15 (two consumer groups of 8 warps): group g takes the CTA's
//     tiles g, g+2, g+4, ... (stage s always belongs to group s % 2). Each
//     8-lane quarter-warp owns RPG rows of a tile, holds its query chunks in
//     registers (the query is quantized in shared memory first, bit-identical
//     to quantizeRowInt8) and dots 16-byte row chunks with dp4a; a
//     transpose-reduce leaves one complete row sum per owner lane;
//   * top-K per group: candidates above the group threshold are appended to a
//     shared buffer; when it fills, a bitonic sort keeps the best k and raises
//     the threshold, which is also published to a per-query global threshold
//     (atomicMax) read back every tile. Every threshold is the k-th best key of
//     k real rows, so nothing that can reach the global top-k is dropped;
//   * merge: each CTA merges its two groups' sorted top-k lists; the last CTA
//     of every block of 8 CTAs (ticket counter) merges the block's lists; the
//     last block merges the block lists and writes the final sorted keys. All
//     merges are "top-k of two sorted lists" bitonic networks in shared memory.
#include "fi8_device.cuh"
#include "fi8_scan.cuh"
#include "fi8_select.cuh"

namespace fi8 {

namespace {

constexpr int kGroups = 2;
constexpr int kConsumerThreads = kGroups * kGroupThreads;
constexpr int kBlockThreads = kConsumerThreads + 32;  // + producer warp
constexpr int kConsumerWarps = kConsumerThreads / 32;
constexpr int kMaxStages = 8;
constexpr size_t kSmemBudget = 220 * 1024;
constexpr int kBarConsumers = 3;  // named barrier over the 512 consumer threads

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One 16-byte chunk of a row against the same chunk of the query: four dp4a
// (int8 W8A8 rows) or four popcounts of the XOR (packed sign bits: the
// Hamming distance of linalg/hamming.go:54-73).
template <bool BIN>
__device__ __forceinline__ int chunk_op(const int4 a, const int4 b, int acc) {
  if (BIN) return acc + __popc(a.x ^ b.x) + __popc(a.y ^ b.y) + __popc(a.z ^ b.z) + __popc(a.w ^ b.w);
  acc = __dp4a(a.x, b.x, acc);
  acc = __dp4a(a.y, b.y, acc);
  acc = __dp4a(a.z, b.z, acc);
  return __dp4a(a.w, b.w, acc);
}

// CPL: 16-byte chunks per lane per row (dpad = 128*CPL), 0 = generic pitch.
// RPG: rows per 8-lane quarter-warp per pass; a tile is R = 32*RPG*passes rows.
// BIN: rows are packed sign bits and a row's value is its Hamming distance to
// the query's bits (no scales). Used without TOPK: every row's distance is
// stored (u16) and counted into a (bits+1)-bin histogram, the first pass of
// prefilterHist (ann/flat_binary_prefilter.go:145-178).
template <bool TOPK, int CPL, int RPG, bool BIN>
__global__ void __launch_bounds__(kBlockThreads, 1) scan_kernel(ScanParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t s_full[kMaxStages];
  __shared__ uint64_t s_empty[kMaxStages];
  __shared__ float s_red[kConsumerWarps];
  __shared__ float s_qscale;
  __shared__ int s_count[kGroups];
  __shared__ unsigned long long s_thr[kGroups];
  __shared__ unsigned long long s_local_thr[kGroups];
  __shared__ volatile int s_abort;
  __shared__ int s_gabort[kGroups];
  __shared__ int s_last;

  constexpr int LOGR = RPG == 1 ? 0 : RPG == 2 ? 1 : RPG == 4 ? 2 : 3;
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
  const uint32_t stage_bytes = code_bytes + (BIN ? 0u : (uint32_t)R * 4u);

  unsigned char* stages = smem;
  int8_t* q_s = reinterpret_cast<int8_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* bufs = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes + (size_t)dpad);

  const int64_t my_tiles = (p.ntiles > cta) ? (p.ntiles - cta + G - 1) / G : 0;

  pdl_launch_dependents();
  if (p.gate) {
    // a gated launch: nothing is read or written unless the gate is open
    // (uniform over the grid, so every thread of every CTA returns alike)
    pdl_wait_prior();
    if (*reinterpret_cast<const volatile unsigned int*>(p.gate) == 0u) return;
  }
  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], kGroupThreads / 32);
    }
    fence_mbar_init();
    s_abort = 0;
    for (int g = 0; g < kGroups; g++) {
      s_count[g] = 0;
      s_local_thr[g] = 0;
      s_thr[g] = 0ull;  // read from gthr after the wait below
    }
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ======================= producer warp =======================
    if (lane == 0) {
      int64_t it = 0;
      for (; it < my_tiles; it++) {
        const int s = (int)(it % S);
        if (it >= S && !mbar_wait_bounded(&s_empty[s], (uint32_t)(((it / S) - 1) & 1))) {
          s_abort = 1;
          atomicOr(p.err, 1u);
        }
        if (s_abort) break;
        const int64_t tile = cta + it * G;
        unsigned char* st = stages + (size_t)s * stage_bytes;
        mbar_arrive_expect_tx(&s_full[s], stage_bytes);
        bulk_g2s(st, p.codes + (size_t)tile * code_bytes, code_bytes, &s_full[s]);
        if (!BIN) bulk_g2s(st + code_bytes, p.scales + (size_t)tile * R, (uint32_t)R * 4u, &s_full[s]);
      }
      if (s_abort) {
        // let the copies already issued land before the CTA can exit (bounded)
        for (int64_t j = (it > S ? it - S : 0); j < it; j++)
          mbar_wait_bounded(&s_full[j % S], (uint32_t)((j / S) & 1));
      }
    }
    __syncwarp();
  } else {
    // ======================= consumer groups =======================
    const int g = warp / (kGroupThreads / 32);
    const int gtid = tid - g * kGroupThreads;
    const int gwarp = gtid >> 5;
    const int bar = 1 + g;
    uint64_t* buf = bufs + (TOPK ? (size_t)g * p.cap : 0);

    // the query (and, binary, the zeroed histogram) may come from the kernel
    // just before this one; the producer streams the corpus meanwhile. So
    // does the per-query threshold: the previous scan on this stream resets
    // it in its very last CTA, after this launch's CTAs may have started on
    // SMs that scan has freed, so it is read only after the wait.
    pdl_wait_prior();
    if (TOPK && gtid == 0) s_thr[g] = ld_relaxed_u64(p.gthr + y);
    if (BIN) {
      // the query's packed sign bits, prepared by the caller
      const int8_t* qb = reinterpret_cast<const int8_t*>(p.qbits) + (size_t)y * dpad;
      for (int i = tid; i < dpad; i += kConsumerThreads) q_s[i] = qb[i];
      if (tid == 0) s_qscale = 0.0f;
      if (!TOPK)
        for (int i = tid; i < p.nbins; i += kConsumerThreads) reinterpret_cast<unsigned int*>(bufs)[i] = 0u;
    } else {
    // quantize this CTA's query (quant.go:43-71) into shared memory
    const float* q = p.q + (size_t)y * p.d;
    float m = 0.0f;
    for (int i = tid; i < p.d; i += kConsumerThreads) m = absmax_step(m, q[i]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = absmax_combine(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) s_red[warp] = m;
    named_sync(kBarConsumers, kConsumerThreads);
    if (tid == 0) {
      float mm = 0.0f;
      for (int w = 0; w < kConsumerWarps; w++) mm = absmax_combine(mm, s_red[w]);
      s_red[0] = mm;
    }
    named_sync(kBarConsumers, kConsumerThreads);
    const float maxabs = s_red[0];
    if (maxabs == 0.0f) {
      for (int i = tid; i < dpad; i += kConsumerThreads) q_s[i] = 0;
      if (tid == 0) s_qscale = 0.0f;
    } else {
      const float sc = __fdiv_rn(maxabs, 127.0f);
      const float inv = __fdiv_rn(1.0f, sc);
      for (int i = tid; i < dpad; i += kConsumerThreads) q_s[i] = i < p.d ? quant_code(q[i], inv) : (int8_t)0;
      if (tid == 0) s_qscale = sc;
    }
    }
    named_sync(kBarConsumers, kConsumerThreads);
    const float qscale = s_qscale;

    const int lane8 = lane & 7;
    const int lg = lane >> 3;
    int4 qreg[CPL > 0 ? CPL : 1];
#pragma unroll
    for (int j = 0; j < (CPL > 0 ? CPL : 1); j++)
      if (CPL > 0) qreg[j] = reinterpret_cast<const int4*>(q_s)[lane8 + 8 * j];

    const int rows_per_pass = 32 * RPG;
    const int passes = R / rows_per_pass;
    for (int64_t it = g; it < my_tiles; it += kGroups) {
      const int s = (int)(it % S);
      if (!mbar_wait_bounded(&s_full[s], (uint32_t)((it / S) & 1))) {
        s_abort = 1;
        atomicOr(p.err, 1u);
      }
      const int64_t row0 = (cta + it * G) * (int64_t)R;
      const unsigned char* st = stages + (size_t)s * stage_bytes;
      const float* sc_s = reinterpret_cast<const float*>(st + code_bytes);
      const unsigned long long thr = TOPK ? s_thr[g] : 0ull;
      unsigned long long gt_prefetch = 0ull;
      if (TOPK && gtid == 0) gt_prefetch = ld_relaxed_u64(p.gthr + y);

      for (int pass = 0; pass < passes; pass++) {
        // rows of this quarter-warp: base .. base + RPG - 1
        const int base = pass * rows_per_pass + gwarp * (4 * RPG) + lg * RPG;
        int vals[RPG];
        if (CPL > 0) {
          int acc[RPG][2];
#pragma unroll
          for (int i = 0; i < RPG; i++) acc[i][0] = acc[i][1] = 0;
#pragma unroll
          for (int j = 0; j < (CPL > 0 ? CPL : 1); j++) {
#pragma unroll
            for (int i = 0; i < RPG; i++) {
              const int4 a = reinterpret_cast<const int4*>(st + (size_t)(base + i) * dpad)[lane8 + 8 * j];
              acc[i][j & 1] = chunk_op<BIN>(a, qreg[j], acc[i][j & 1]);
            }
          }
#pragma unroll
          for (int i = 0; i < RPG; i++) vals[i] = acc[i][0] + acc[i][1];
        } else {
          const int chunks = dpad >> 4;
          const int4* rowp = reinterpret_cast<const int4*>(st + (size_t)base * dpad);
          const int4* qp = reinterpret_cast<const int4*>(q_s);
          int a0 = 0, a1 = 0;
          int c = lane8;
          for (; c + 8 < chunks; c += 16) {
            const int4 a = rowp[c], b = qp[c];
            const int4 a2 = rowp[c + 8], b2 = qp[c + 8];
            a0 = chunk_op<BIN>(a, b, a0);
            a1 = chunk_op<BIN>(a2, b2, a1);
          }
          if (c < chunks) {
            const int4 a = rowp[c], b = qp[c];
            a0 = chunk_op<BIN>(a, b, a0);
          }
          vals[0] = a0 + a1;
        }
        // transpose-reduce over the 8 lanes: lane8 >> (3-LOGR) ends up owning
        // row (base + that index) with the complete sum.
#pragma unroll
        for (int h = RPG, off = 4; h > 1; h >>= 1, off >>= 1) {
          const bool upper = (lane8 & off) != 0;
#pragma unroll
          for (int t = 0; t < h / 2; t++) {
            const int keep = upper ? vals[t + h / 2] : vals[t];
            const int send = upper ? vals[t] : vals[t + h / 2];
            vals[t] = keep + __shfl_xor_sync(0xffffffffu, send, off);
          }
        }
#pragma unroll
        for (int off = 4 >> LOGR; off >= 1; off >>= 1) vals[0] += __shfl_xor_sync(0xffffffffu, vals[0], off);

        const bool owner = (lane8 & ((8 >> LOGR) - 1)) == 0;
        const int r = base + (lane8 >> (3 - LOGR));
        const int64_t gr = row0 + r;
        const bool mine = owner && (gr < p.n);
        const bool kept = mine && (!p.keep || keep_bit(p.keep, p.keep_nbits, p.id_base + (uint64_t)gr));
        float score = 0.0f;
        if (mine) score = BIN ? (float)(-vals[0]) : w8a8_score(vals[0], qscale, sc_s[r]);
        if (TOPK) {
          uint64_t key = kEmptyKey;
          bool take = false;
          if (kept && score == score) {
            key = make_key(score, p.id_base + (uint32_t)gr);
            take = key > thr;
          }
          warp_append(take, key, buf, &s_count[g]);
        } else if (mine) {
          if (BIN) {
            // a filtered-out row gets a distance above every cut and no count
            p.out_dist[(size_t)y * p.dist_stride + gr] = kept ? (uint16_t)vals[0] : (uint16_t)0xFFFFu;
            if (kept) atomicAdd(reinterpret_cast<unsigned int*>(bufs) + vals[0], 1u);
          } else {
            p.out_scores[(size_t)y * p.n + gr] = score;
          }
        }
      }
      // this warp is done reading the stage
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[s]);
      if (TOPK) {
        named_sync(bar, kGroupThreads);
        const int cnt = s_count[g];
        if (cnt > p.cap - R) group_compact(buf, cnt, p.k, &s_count[g], &s_local_thr[g], p.gthr + y, gtid, bar);
        if (gtid == 0) {
          s_thr[g] = gt_prefetch > s_local_thr[g] ? gt_prefetch : s_local_thr[g];
          s_gabort[g] = s_abort;
        }
        named_sync(bar, kGroupThreads);
        if (s_gabort[g]) break;  // group-uniform: read after the barrier
      } else if (__any_sync(0xffffffffu, s_abort)) {
        break;  // warp-uniform (score mode has no group barriers)
      }
    }
    if (TOPK) {
      named_sync(bar, kGroupThreads);
      group_compact(buf, s_count[g], p.k, &s_count[g], &s_local_thr[g], p.gthr + y, gtid, bar);
      // the group's list: its best keys, sorted, empty-padded to kp
      for (int i = s_count[g] + gtid; i < p.kp; i += kGroupThreads) buf[i] = kEmptyKey;
    }
    if (BIN && !TOPK) {
      // this CTA's histogram into the query's
      named_sync(kBarConsumers, kConsumerThreads);
      const unsigned int* hs = reinterpret_cast<const unsigned int*>(bufs);
      for (int b = tid; b < p.nbins; b += kConsumerThreads)
        if (hs[b]) atomicAdd(p.hist + (size_t)y * p.nbins + b, hs[b]);
    }
  }

  if (!TOPK) return;
  __syncthreads();  // both groups (and the producer) are done
  const int kp = p.kp;
  const int NB = (G + kMergeBlock - 1) / kMergeBlock;
  if (warp < kGroupThreads / 32) {
    // group 0 merges the two group lists of this CTA. They sit cap keys apart;
    // group 1's list moves next to group 0's (kp <= cap/2 unless kp == cap, in
    // which case the copy is in place, so source and target never overlap).
    for (int i = tid; i < kp; i += kGroupThreads) bufs[kp + i] = bufs[(size_t)p.cap + i];
    named_sync(1, kGroupThreads);
    tree_merge_slots(bufs, 2, kp, tid, 1);
    uint64_t* mine = p.lvl1 + ((size_t)y * G + cta) * kp;
    for (int i = tid; i < kp; i += kGroupThreads) mine[i] = bufs[i];
    __threadfence();
  }
  __syncthreads();
  const int blk = cta / kMergeBlock;
  const int members = min(kMergeBlock, G - blk * kMergeBlock);
  if (tid == 0) {
    const unsigned int ticket = atomicAdd(p.counter + (size_t)y * NB + blk, 1u);
    s_last = (ticket == (unsigned int)(members - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (!s_last || warp >= kGroupThreads / 32) return;

  // ---- last CTA of the block: merge the block's CTA lists ----
  __threadfence();
  const int nslots = p.smem_bytes / (kp * 8);
  uint64_t* slots = reinterpret_cast<uint64_t*>(smem);
  merge_global_lists(p.lvl1 + ((size_t)y * G + (size_t)blk * kMergeBlock) * kp, members, kp, kp, kp, slots,
                     nslots, tid, 1);
  uint64_t* blist = p.lvl2 + ((size_t)y * NB + blk) * kp;
  for (int i = tid; i < kp; i += kGroupThreads) blist[i] = slots[i];
  if (tid == 0) p.counter[(size_t)y * NB + blk] = 0u;  // every member has taken its ticket
  __threadfence();
  named_sync(1, kGroupThreads);
  if (tid == 0) {
    const unsigned int ticket = atomicAdd(p.counter2 + y, 1u);
    s_last = (ticket == (unsigned int)(NB - 1)) ? 1 : 0;
  }
  named_sync(1, kGroupThreads);
  if (!s_last) return;

  // ---- last block: merge the block lists, write the final keys ----
  __threadfence();
  merge_global_lists(p.lvl2 + (size_t)y * NB * kp, NB, kp, kp, kp, slots, nslots, tid, 1);
  for (int i = tid; i < p.k; i += kGroupThreads) p.out_keys[(size_t)y * p.k + i] = slots[i];
  if (tid == 0) {
    p.counter2[y] = 0u;
    p.gthr[y] = 0ull;
  }
}

// ---------------------------------------------------------------------------
// merge_keys_kernel: top-k of nsrc sorted candidate lists per query, one CTA
// each. The cross-GPU merge after the all-gather (the N-way analogue of
// queryBatchSharded's merge, ann/backend.go:262-277).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kGroupThreads, 1)
    merge_keys_kernel(const uint64_t* in, int nsrc, int M, int k, int kp, int nslots, uint64_t* out) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* slots = reinterpret_cast<uint64_t*>(smem);
  const int y = blockIdx.x;
  pdl_launch_dependents();
  pdl_wait_prior();
  merge_global_lists(in + (size_t)y * k, nsrc, k, (size_t)M * k, kp, slots, nslots, threadIdx.x, 1);
  for (int i = threadIdx.x; i < k; i += kGroupThreads) out[(size_t)y * k + i] = slots[i];
}

int pow2_at_least(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

using ScanFn = void (*)(ScanParams);

// (CPL, RPG) pairs with a specialised kernel; RPG keeps a pass near 24-32 KB.
struct Shape {
  int cpl, rpg;
};
constexpr Shape kShapes[] = {{1, 8}, {2, 4}, {3, 2}, {4, 2}, {6, 1}, {8, 1}, {12, 1}, {16, 1}};

template <bool TOPK>
ScanFn pick_kernel(int cpl) {
  switch (cpl) {
    case 1: return scan_kernel<TOPK, 1, 8, false>;
    case 2: return scan_kernel<TOPK, 2, 4, false>;
    case 3: return scan_kernel<TOPK, 3, 2, false>;
    case 4: return scan_kernel<TOPK, 4, 2, false>;
    case 6: return scan_kernel<TOPK, 6, 1, false>;
    case 8: return scan_kernel<TOPK, 8, 1, false>;
    case 12: return scan_kernel<TOPK, 12, 1, false>;
    case 16: return scan_kernel<TOPK, 16, 1, false>;
    default: return scan_kernel<TOPK, 0, 1, false>;
  }
}

// Packed sign bits (histogram mode): 128-byte rows (d in (960, 1024]) and
// 256-byte rows get specialised kernels, every other pitch the generic one.
ScanFn pick_binary_kernel(int cpl) {
  switch (cpl) {
    case 1: return scan_kernel<false, 1, 8, true>;
    case 2: return scan_kernel<false, 2, 4, true>;
    default: return scan_kernel<false, 0, 1, true>;
  }
}

int rows_per_group(int dpad, bool binary, int* cpl_out) {
  *cpl_out = 0;
  if (dpad % 128 == 0)
    for (const Shape& s : kShapes)
      if (s.cpl * 128 == dpad && (!binary || s.cpl <= 2)) {
        *cpl_out = s.cpl;
        return s.rpg;
      }
  return 1;
}

}  // namespace

bool scan_geometry(int32_t dpad, int32_t k, bool topk, ScanGeometry* g, bool binary) {
  if (dpad <= 0 || dpad % 16 != 0 || dpad > kScanMaxDpad) return false;
  if (binary && topk) return false;
  int cpl = 0;
  const int rpg = rows_per_group(dpad, binary, &cpl);
  const size_t row_bytes = (size_t)dpad + (binary ? 0 : 4);
  int cap = 0, kp = 0;
  if (topk) {
    if (k <= 0) return false;
    // room for k survivors plus one tile of new candidates between compactions
    cap = pow2_at_least(k + 256);
    kp = pow2_at_least(k);
    if (cap > kScanMaxCap) return false;
  }
  // query row, then the groups' candidate buffers (top-K) or the distance
  // histogram of dpad*8 + 1 bins (binary)
  const size_t fixed = (size_t)dpad + (size_t)kGroups * cap * 8 + (binary ? ((size_t)dpad * 8 + 1) * 4 : 0);
  // Tile (R rows, a power-of-two multiple of one pass of 32*RPG rows, at most
  // 256 so it divides the allocation padding) and ring depth S (even: stage s
  // always belongs to consumer group s % 2; with an odd count the groups would
  // share stages, and because bulk copies complete out of order a parity wait
  // could then observe the wrong phase). One CTA per SM moves a bounded number
  // of copies per second, so tiles must be large; measured on B200 (C2-size
  // corpora, 768-1024-byte and 256-384-byte rows): 32 KB x 4 and ~96 KB x 2
  // sustain ~7.0 TB/s, 48-64 KB tiles 6.7-6.9, 24 KB x 6 only 6.2.
  struct Choice {
    int R, S;
  } pick[3];
  int np = 0;
  for (int r = 32 * rpg; r <= 256; r *= 2)
    if ((size_t)r * dpad == 32 * 1024) pick[np++] = {r, 4};
  {
    int r = 32 * rpg;
    while (r < 256 && (size_t)(2 * r) * dpad <= 100 * 1024) r *= 2;
    if ((size_t)r * dpad >= 48 * 1024) pick[np++] = {r, 2};
  }
  {
    int r = 32 * rpg;  // small rows: the largest tile at or under 32 KB, deeper ring
    while (r < 256 && (size_t)(2 * r) * dpad <= 32 * 1024) r *= 2;
    int st = 2;
    while (st + 2 <= kMaxStages && (size_t)(st + 2) * r * row_bytes <= 160 * 1024) st += 2;
    pick[np++] = {r, st};
  }
  int R = 0, stages = 0;
  for (int i = 0; i < np && !R; i++)
    for (int st = pick[i].S; st >= 2 && !R; st -= 2)
      if (fixed + (size_t)st * pick[i].R * row_bytes <= kSmemBudget) {
        R = pick[i].R;
        stages = st;
      }
  if (!R) return false;
  const size_t stage = (size_t)R * row_bytes;
  g->rows_per_tile = R;
  g->stages = stages;
  g->cap = cap;
  g->kp = kp;
  g->smem_bytes = fixed + stages * stage;
  // the merges reuse the dynamic shared memory for lists of kp keys: at least
  // two must fit
  if (topk && g->smem_bytes < (size_t)2 * kp * 8) g->smem_bytes = (size_t)2 * kp * 8;
  return true;
}

cudaError_t scan_launch(const ScanParams& p, bool topk, int32_t M, int32_t G, cudaStream_t stream, bool binary) {
  if (p.stages > kMaxStages || p.stages % kGroups != 0 || p.stages < 2) return cudaErrorInvalidValue;
  if (binary && (topk || !p.qbits || !p.hist || !p.out_dist || p.nbins != p.dpad * 8 + 1))
    return cudaErrorInvalidValue;
  int cpl = 0;
  const int rpg = rows_per_group(p.dpad, binary, &cpl);
  if (p.rows_per_tile % (32 * rpg) != 0) return cudaErrorInvalidValue;
  ScanFn fn = binary ? pick_binary_kernel(cpl) : topk ? pick_kernel<true>(cpl) : pick_kernel<false>(cpl);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)G, (unsigned)M);
  if (binary || p.gate)  // follows the query packing kernel, or a gated redo chain
    return launch_pdl(fn, grid, dim3(kBlockThreads), (size_t)p.smem_bytes, stream, p);
  void* args[] = {const_cast<ScanParams*>(&p)};
  return cudaLaunchKernel(reinterpret_cast<const void*>(fn), grid, dim3(kBlockThreads), args,
                          (size_t)p.smem_bytes, stream);
}

cudaError_t merge_keys_launch(const uint64_t* in, int32_t nsrc, int32_t M, int32_t k, uint64_t* out,
                              cudaStream_t stream, bool pdl) {
  if (k <= 0 || k > kMergeMaxK || nsrc <= 0 || M <= 0) return cudaErrorInvalidValue;
  const int kp = pow2_at_least(k);
  int nslots = (int)(kSmemBudget / ((size_t)kp * 8));
  if (nslots > nsrc + 1) nslots = nsrc + 1;
  if (nslots < 2) nslots = 2;
  cudaError_t e = cudaFuncSetAttribute(merge_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBudget);
  if (e != cudaSuccess) return e;
  if (pdl)
    return launch_pdl(merge_keys_kernel, dim3((unsigned)M), dim3(kGroupThreads), (size_t)nslots * kp * 8, stream, in,
                      nsrc, M, k, kp, nslots, out);
  merge_keys_kernel<<<M, kGroupThreads, (size_t)nslots * kp * 8, stream>>>(in, nsrc, M, k, kp, nslots, out);
  return cudaGetLastError();
}

}  // namespace fi8
