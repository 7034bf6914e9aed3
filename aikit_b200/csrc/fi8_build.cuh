// fi8_build.cuh -- host-visible declarations for the device corpus build
// (NewFlatI8's quantization, newBinaryPrefilter's centring and packing).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace fi8 {

// codes[r][0..dpad) and scales[r] for rows v[r][0..dim) of a chunk, as
// QuantizeRowInt8 with an all-zero row taking scale 1.
cudaError_t quantize_rows_launch(const float* v, int64_t rows, int32_t dim, int32_t dpad, int8_t* codes,
                                 float* scales, cudaStream_t stream);

// acc[j] += v[r][j] over the chunk's rows whose valid byte is non-zero (valid
// may be null), in row order, in float64: call once per chunk, in order.
cudaError_t column_sum_launch(const float* v, int64_t rows, int32_t dim, const uint8_t* valid, double* acc,
                              cudaStream_t stream);

// center[j] = float32(acc[j] / used).
cudaError_t center_launch(const double* acc, int32_t dim, int64_t used, float* center, cudaStream_t stream);

// bits[r][0..wpad) = PackSignBitsRow(v[r] - center) (center may be null);
// rows whose valid byte is 0 stay all-zero.
cudaError_t pack_rows_launch(const float* v, int64_t rows, int32_t dim, const float* center, const uint8_t* valid,
                             int32_t wpad, uint64_t* bits, cudaStream_t stream);

}  // namespace fi8
