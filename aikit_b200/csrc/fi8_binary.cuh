// fi8_binary.cuh -- host-visible declarations for the FlatBinaryI8 device path:
// query sign-bit packing and the int8 rerank of a Hamming shortlist. The
// Hamming scan itself is the scan kernel's binary mode (fi8_scan.cuh).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace fi8 {

// qbits[y][w] = the packed sign bits of (q[y] - center) (center may be null):
// bit i%64 of word i/64 is set iff q[y][i] - center[i] >= 0 in float32, bits
// past d and words past ceil(d/64) are zero. wpad = row pitch in words.
cudaError_t binary_prep_launch(const float* q, int32_t M, int32_t d, const float* center, int32_t wpad,
                               uint64_t* qbits, cudaStream_t stream);

// Exact W8A8 top-k over a shortlist: for each query y, the entries of
// shortlist[y][0..cand) (packed keys whose index is a global row id; 0 =
// empty) that fall in this shard's rows [id_base, id_base + n) are scored
// against codes/scales (dpad pitch) exactly as the scan scores them, and
// out[y][0..k) receives the best k keys, sorted, 0-padded.
cudaError_t rerank_launch(const float* q, int32_t M, int32_t d, int32_t dpad, const int8_t* codes,
                          const float* scales, int64_t n, uint32_t id_base, const uint64_t* shortlist,
                          int32_t cand, int32_t k, uint64_t* out, cudaStream_t stream);

// Largest shortlist (cand) the rerank sorts in shared memory.
constexpr int32_t kRerankMaxCand = 4096;

}  // namespace fi8
