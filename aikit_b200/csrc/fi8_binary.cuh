// fi8_binary.cuh -- host-visible declarations for the FlatBinaryI8 device path:
// query sign-bit packing, the prefilter's shortlist from the distance
// histogram, and the int8 rerank of the shortlist. The distance pass itself is
// the scan kernel's binary histogram mode (fi8_scan.cuh).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace fi8 {

// qbits[y][w] = the packed sign bits of (q[y] - center) (center may be null):
// bit i%64 of word i/64 is set iff q[y][i] - center[i] >= 0 in float32, bits
// past d are zero; wpad = row pitch in words. Also zeroes hist[y][0..nbins).
// gate (optional): the launch does nothing unless *gate != 0 (the exact redo
// of a tensor-core shortlist that dropped candidates).
cudaError_t binary_prep_launch(const float* q, int32_t M, int32_t d, const float* center, int32_t wpad,
                               uint64_t* qbits, unsigned int* hist, int32_t nbins, cudaStream_t stream,
                               const unsigned int* gate = nullptr);

// Row segments the shortlist kernels split a corpus into (counts holds
// [M][P][2] entries).
int32_t shortlist_segments(int32_t sm_count);

// From each query's distances dist[y][0..n) (row stride dstride, a multiple of
// 8) and histogram hist[y][0..nbins): out[y][0..cand) = packed keys
// (-distance, id_base + row) of prefilterHist's cand rows -- every row below
// the cut t, then the first ties at t in id order -- 0 past the rows there
// are. sorted: also sort each query's keys descending (for a key merge).
// gate as for binary_prep_launch.
cudaError_t shortlist_launch(const uint16_t* dist, int64_t n, int64_t dstride, int32_t M, const unsigned int* hist,
                             int32_t nbins, int32_t cand, int32_t P, unsigned int* counts, uint32_t id_base,
                             uint64_t* out, bool sorted, cudaStream_t stream, const unsigned int* gate = nullptr);

// CTAs (slices of the shortlist) one query's rerank uses; parts holds
// [rerank_parts(cand)][M][k] keys.
int32_t rerank_parts(int32_t cand);

// Exact W8A8 top-k over a shortlist: for each query y, the entries of
// shortlist[y][0..cand) (packed keys whose index is a global row id; 0 =
// empty) that fall in this shard's rows [id_base, id_base + n) are scored
// against codes/scales (dpad pitch) exactly as the scan scores them, and
// out[y][0..k) receives the best k keys, sorted, 0-padded.
cudaError_t rerank_launch(const float* q, int32_t M, int32_t d, int32_t dpad, const int8_t* codes,
                          const float* scales, int64_t n, uint32_t id_base, const uint64_t* shortlist,
                          int32_t cand, int32_t k, uint64_t* parts, uint64_t* out, cudaStream_t stream);

// The codes unpacked for the tensor-core prefilter: rows[r][i] = +1 where bit
// i of row r's code is set, -1 where it is clear (i < d), 0 for i >= d and
// for rows r >= n (n_alloc rows of dpad bytes; dpad a multiple of 16).
cudaError_t sign_rows_launch(const uint64_t* bits, int64_t n, int64_t n_alloc, int32_t wpad, int32_t d, int32_t dpad,
                             int8_t* rows, cudaStream_t stream);

// Largest shortlist (cand) the shortlist sort and the rerank support.
constexpr int32_t kRerankMaxCand = 4096;

}  // namespace fi8
