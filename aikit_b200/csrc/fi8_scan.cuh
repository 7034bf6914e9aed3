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
  int32_t rows_per_tile; // R, multiple of 32, divides 256
  int32_t stages;        // bulk-copy pipeline depth
  int64_t ntiles;        // n_alloc / R
  const float* q;        // [M][d] f32 queries
  uint32_t id_base;      // global id of row 0 (row sharding)
  // top-K mode
  int32_t k;
  int32_t cap;           // candidate buffer (power of two, >= k + R)
  unsigned long long* gthr;  // [M] shared per-query threshold key (zero at rest)
  unsigned int* counter;     // [M] CTA completion tickets (zero at rest)
  uint64_t* part_keys;       // [M][L][k] surviving keys per list (L = 2G)
  int32_t* part_counts;      // [M][L]
  uint64_t* out_keys;        // [M][k] final keys, 0 = empty
  // score mode
  float* out_scores;         // [M][n]
  unsigned int* err;         // device error flags (bit 0: wait timeout)
};

struct ScanGeometry {
  int32_t rows_per_tile;
  int32_t stages;
  int32_t cap;
  size_t smem_bytes;
};

// Largest supported row pitch and top-K for the scan kernels.
constexpr int32_t kScanMaxDpad = 2048;
constexpr int32_t kScanMaxCap = 4096;

bool scan_geometry(int32_t dpad, int32_t k, bool topk, ScanGeometry* g);
cudaError_t scan_launch(const ScanParams& p, bool topk, int32_t M, int32_t G, size_t smem,
                        cudaStream_t stream);

// Survivor lists per query of a top-K scan launched with G CTAs (each CTA
// runs two consumer groups, each with its own list).
int32_t scan_lists_per_query(int32_t G);
// Scratch sizes (elements) for a top-K scan over M queries with G CTAs each.
inline size_t scan_part_keys(int32_t M, int32_t G, int32_t k) {
  return (size_t)M * scan_lists_per_query(G) * k;
}

// Merge nsrc sorted-or-unsorted key lists per query ([nsrc][M][k], 0 = empty)
// into the top k per query ([M][k]). One CTA per query.
cudaError_t merge_keys_launch(const uint64_t* in, int32_t nsrc, int32_t M, int32_t k,
                              uint64_t* out, cudaStream_t stream);
constexpr int32_t kMergeMaxK = 2048;

}  // namespace fi8
