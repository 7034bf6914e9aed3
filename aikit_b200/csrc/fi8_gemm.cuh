// fi8_gemm.cuh -- host-visible declarations for the batched FlatI8 path:
// query quantization, the tcgen05 kind::i8 GEMM with a threshold-filter
// epilogue, and the per-query exact select between row ranges.
#pragma once

#include <cuda.h>
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace fi8 {

constexpr int32_t kGemmBM = 128;  // largest query tile (TMEM lanes); 64 for batches of <= 64
constexpr int32_t kGemmBN = 256;  // corpus rows per tile (MMA N)
constexpr int32_t kGemmBK = 128;  // K bytes per pipeline stage (one 128B-swizzle row)

struct GemmLevel {
  int64_t row_lo, row_hi;  // corpus rows [lo, hi) of this range; lo % 256 == 0
};

struct GemmParams {
  int64_t row_lo, row_hi;
  int32_t kchunks;       // ceil(dpad / 128)
  int32_t M;             // real queries
  int32_t qtiles;        // ceil(M / 128)
  int64_t rtiles;        // 256-row tiles in [row_lo, row_hi)
  uint32_t id_base;      // global id of corpus row 0
  const float* scales;   // [n_alloc] row scales (W8A8 mode)
  int32_t ham_dim;       // > 0: Hamming mode -- A and B are +1/-1 sign rows
                         // (0 past ham_dim) and a row's score is -(Hamming
                         // distance) = (dot - ham_dim) / 2; 0: W8A8 scores
  const float* qscale;   // [Mpad] query scales
  const unsigned long long* thr;  // [M] per-query threshold key (0 = none)
  unsigned int* cnt;     // [M] candidates appended this range
  uint64_t* cand;        // [M][cap] candidate keys
  int32_t cap;
  unsigned int* err;
  int32_t producer_waits;  // 1: the producer waits for the previous kernel (it wrote A)
  const uint64_t* keep;    // optional keep bitmap over global ids
  int64_t keep_nbits;
};

// Build a 2-D SWIZZLE_128B tensor map over an int8 matrix [rows][pitch]
// (pitch a multiple of 16 bytes) with a {128 bytes, box_rows} box.
bool make_tmap_i8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t pitch, uint32_t box_rows);

// bm: the query tile (64 or 128); tmA's box must be bm rows. pair: clusters
// of two CTAs (tcgen05 cta_group::2) over 256-query x 256-row units; then bm
// is 128, G (CTAs) and p.qtiles are even, and tmB's box is 128 rows (each CTA
// loads half of a unit's corpus rows); otherwise tmB's box is 256 rows.
cudaError_t gemm_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p, int32_t G, int32_t bm,
                        bool pair, cudaStream_t stream);

// Clusters of two GEMM CTAs that can be resident at once on this device (0 if
// the pair form cannot launch).
int32_t gemm_pair_max_clusters();

// Quantize M queries ([M][d] f32) into A ([Mpad][dpad] int8, zero padded) and
// qscale ([Mpad]); also resets the per-query select state (thr, cnt, topk).
cudaError_t quantize_launch(const float* q, int32_t M, int32_t Mpad, int32_t d, int32_t dpad, int8_t* A,
                            float* qscale, unsigned long long* thr, unsigned int* cnt, uint64_t* topk, int32_t kp,
                            int32_t bm, cudaStream_t stream);

// The Hamming mode's A: query j's sign row, +1 where q[j][i] - center[i] >= 0
// in float32 (center may be null), -1 elsewhere (NaN included), 0 past d;
// qscale 1 (0 for rows without a query); the select state reset as above.
cudaError_t sign_prep_launch(const float* q, int32_t M, int32_t Mpad, int32_t d, int32_t dpad, const float* center,
                             int8_t* A, float* qscale, unsigned long long* thr, unsigned int* cnt, uint64_t* topk,
                             int32_t kp, int32_t bm, cudaStream_t stream);

// Per query: top-k of (carried topk list [kp] U this range's candidates) ->
// topk, thr = k-th best key (0 if fewer), cnt = 0; optionally out[q][k].
cudaError_t select_launch(int32_t M, int32_t k, int32_t kp, uint64_t* topk, unsigned long long* thr,
                          unsigned int* cnt, const uint64_t* cand, int32_t cap, uint64_t* out, unsigned int* err,
                          int32_t sm_count, cudaStream_t stream);

int32_t select_max_k();

// After a batch's last select: *gate = whether a select dropped candidates
// (err bit 1), and that bit cleared. A gated redo launch follows it.
cudaError_t overflow_latch_launch(unsigned int* err, unsigned int* gate, cudaStream_t stream);

// Tensor-pipe probe: G CTAs (one per SM) issue iters x 4 back-to-back
// kind::i8 MMAs (M=128, N=256, K=32) on shared-memory operands; ops done.
cudaError_t mma_probe_launch(int32_t G, int64_t iters, unsigned int* err, cudaStream_t stream);
double mma_probe_ops(int32_t G, int64_t iters);

}  // namespace fi8
