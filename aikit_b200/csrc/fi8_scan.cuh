// fi8_scan.cuh -- host-visible declarations for the streaming W8A8 scan
// kernels (batch-1 GEMV form) and the key-merge kernel.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace fi8 {

// Everything one scan launch needs. Device pointers unless noted.
struct ScanParams {
  const int8_t* codes;   // [n_alloc][dpad] int8, rows zero-padded to dpad
  const float* scales;   // [n_alloc] f32, zero past n
  int64_t n;             // real rows
  int32_t d;             // query length (reference dim)
  int32_t dpad;          // row pitch in bytes, multiple of 16
  int32_t rows_per_tile; // R, power of two in [32, 256]
  int32_t stages;        // bulk-copy ring depth (even)
  int64_t ntiles;        // n_alloc / R
  const float* q;        // [M][d] f32 queries
  uint32_t id_base;      // global id of row 0 (row sharding)
  const uint64_t* keep;  // optional keep bitmap over global ids (top-K and binary modes)
  int64_t keep_nbits;
  int32_t smem_bytes;    // dynamic shared memory of the launch
  // top-K mode
  int32_t k;
  int32_t kp;            // k rounded up to a power of two: length of every list
  int32_t cap;           // per-group candidate buffer (power of two, >= k + 256)
  unsigned long long* gthr;  // [M] shared per-query threshold key (zero at rest)
  unsigned int* counter;     // [M][NB] per-block CTA tickets (zero at rest)
  unsigned int* counter2;    // [M] block tickets (zero at rest)
  uint64_t* lvl1;            // [M][G][kp] per-CTA top-kp lists
  uint64_t* lvl2;            // [M][NB][kp] per-block top-kp lists
  uint64_t* out_keys;        // [M][k] final keys, 0 = empty
  // binary (packed sign bit) histogram mode: codes are [n_alloc][dpad] bytes
  // of packed bits, scales unused, qbits holds each query's packed bits
  const uint64_t* qbits;     // [M][dpad / 8]
  uint16_t* out_dist;        // [M][dist_stride] Hamming distances
  int64_t dist_stride;
  unsigned int* hist;        // [M][nbins] distance counts (accumulated into)
  int32_t nbins;             // dpad * 8 + 1
  // score mode
  float* out_scores;         // [M][n]
  unsigned int* err;         // device error flags (bit 0: wait timeout)
  // optional gate: when set, the launch runs only if *gate != 0 (read after
  // the previous kernel on the stream completes); otherwise every CTA
  // returns at once. The batched path's exact redo after a dropped
  // candidate is such a launch.
  const unsigned int* gate;
};

struct ScanGeometry {
  int32_t rows_per_tile;
  int32_t stages;
  int32_t cap;
  int32_t kp;
  size_t smem_bytes;
};

// Largest supported row pitch and candidate buffer for the scan kernels.
constexpr int32_t kScanMaxDpad = 2048;
constexpr int32_t kScanMaxCap = 4096;
// CTAs whose lists one first-level merge combines.
constexpr int32_t kMergeBlock = 8;

bool scan_geometry(int32_t dpad, int32_t k, bool topk, ScanGeometry* g, bool binary = false);
cudaError_t scan_launch(const ScanParams& p, bool topk, int32_t M, int32_t G, cudaStream_t stream,
                        bool binary = false);

inline int32_t scan_blocks(int32_t G) { return (G + kMergeBlock - 1) / kMergeBlock; }

// Merge nsrc key lists per query ([nsrc][M][k], each sorted descending, 0 =
// empty) into the top k per query ([M][k]). One CTA per query.
// pdl: launched as a programmatic dependent of the kernel before it.
cudaError_t merge_keys_launch(const uint64_t* in, int32_t nsrc, int32_t M, int32_t k,
                              uint64_t* out, cudaStream_t stream, bool pdl = false);
constexpr int32_t kMergeMaxK = 2048;

}  // namespace fi8
