// fi8_build.cu -- corpus build on the device: NewFlatI8's row quantization
// and newBinaryPrefilter's centring and sign packing, bit-identical to the
// reference's CPU build.
//
// Reference: NewFlatI8 -> QuantizeRowInt8 (ann/flat_i8.go:74-109,
// linalg/quant.go:43-71, all-zero row -> scale 1); newBinaryPrefilter
// (ann/flat_binary_prefilter.go:57-108): center[i] = float32(float64 sum of
// the valid rows' v[i], in row order / used), codes = PackSignBitsRow(v -
// center), invalid (ragged) rows excluded from the sum and left all-zero.
//
// The float64 sum is order-dependent, so it keeps the reference's order: one
// thread per column adds the rows one after another (each chunk of rows after
// the previous one).
#include "fi8_build.cuh"
#include "fi8_device.cuh"

namespace fi8 {

namespace {

constexpr int kRowWarps = 8;  // rows per 256-thread CTA (a warp per row)

// A warp per row: max |v| (NaN ignored), the scale and the codes at pitch dpad.
__global__ void __launch_bounds__(kRowWarps * 32) quantize_rows_kernel(const float* v, int64_t rows, int dim,
                                                                       int dpad, int8_t* codes, float* scales) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* row = v + (size_t)r * dim;
  float m = 0.0f;
  for (int i = lane; i < dim; i += 32) m = absmax_step(m, row[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = absmax_combine(m, __shfl_xor_sync(0xffffffffu, m, off));
  int8_t* out = codes + (size_t)r * dpad;
  if (m == 0.0f) {  // all-zero row: codes 0, scale 1 (quant.go:53-57 with zero scale 1)
    for (int i = lane; i < dpad; i += 32) out[i] = 0;
    if (lane == 0) scales[r] = 1.0f;
    return;
  }
  const float sc = __fdiv_rn(m, 127.0f);
  const float inv = __fdiv_rn(1.0f, sc);
  for (int i = lane; i < dpad; i += 32) out[i] = i < dim ? quant_code(row[i], inv) : (int8_t)0;
  if (lane == 0) scales[r] = sc;
}

// Column sums in the reference's order. A CTA owns 32 columns; warp 0 (a
// thread per column) adds the rows one after another from shared memory while
// warps 1-7 stage the next 128-row tile (128 bytes of each row, coalesced).
// The float64 add chain per column is the limit, so the column slabs run on
// separate SMs.
constexpr int kSumRows = 128;
__global__ void __launch_bounds__(256) column_sum_kernel(const float* v, int64_t rows, int dim, const uint8_t* valid,
                                                         double* acc) {
  __shared__ float tile[2][kSumRows][32];
  __shared__ uint8_t ok[2][kSumRows];
  const int c0 = blockIdx.x * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t ntiles = (rows + kSumRows - 1) / kSumRows;
  auto stage = [&](int64_t t, int b) {  // warps 1-7
    const int64_t r0 = t * kSumRows;
    for (int idx = tid - 32; idx < kSumRows * 32; idx += 224) {
      const int rr = idx >> 5, cc = idx & 31;
      const int64_t r = r0 + rr;
      tile[b][rr][cc] = (r < rows && c0 + cc < dim) ? __ldg(v + (size_t)r * dim + c0 + cc) : 0.0f;
      if (cc == 0) ok[b][rr] = (r < rows) && (!valid || valid[r]);
    }
  };
  double s = (warp == 0 && c0 + lane < dim) ? acc[c0 + lane] : 0.0;
  if (warp > 0 && ntiles > 0) stage(0, 0);
  __syncthreads();
  for (int64_t t = 0; t < ntiles; t++) {
    const int b = (int)(t & 1);
    if (warp == 0) {
      for (int rr = 0; rr < kSumRows; rr++)
        if (ok[b][rr]) s = __dadd_rn(s, (double)tile[b][rr][lane]);
    } else if (t + 1 < ntiles) {
      stage(t + 1, b ^ 1);
    }
    __syncthreads();
  }
  if (warp == 0 && c0 + lane < dim) acc[c0 + lane] = s;
}

__global__ void center_kernel(const double* acc, int dim, int64_t used, float* center) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j < dim) center[j] = (float)__ddiv_rn(acc[j], (double)used);
}

// A warp per row: bit i%64 of word i/64 = (v[i] - center[i]) >= 0; invalid
// rows and bits past dim are 0.
__global__ void __launch_bounds__(kRowWarps * 32) pack_rows_kernel(const float* v, int64_t rows, int dim,
                                                                   const float* center, const uint8_t* valid,
                                                                   int wpad, uint64_t* bits) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* row = v + (size_t)r * dim;
  uint32_t* out = reinterpret_cast<uint32_t*>(bits + (size_t)r * wpad);
  const bool ok = !valid || valid[r];
  for (int base = 0; base < wpad * 64; base += 32) {
    const int i = base + lane;
    bool bit = false;
    if (ok && i < dim) {
      float x = row[i];
      if (center) x = __fsub_rn(x, center[i]);
      bit = x >= 0.0f;
    }
    const uint32_t m = __ballot_sync(0xffffffffu, bit);
    if (lane == 0) out[base >> 5] = m;
  }
}

}  // namespace

cudaError_t quantize_rows_launch(const float* v, int64_t rows, int32_t dim, int32_t dpad, int8_t* codes,
                                 float* scales, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const unsigned grid = (unsigned)((rows + kRowWarps - 1) / kRowWarps);
  quantize_rows_kernel<<<grid, kRowWarps * 32, 0, stream>>>(v, rows, dim, dpad, codes, scales);
  return cudaGetLastError();
}

cudaError_t column_sum_launch(const float* v, int64_t rows, int32_t dim, const uint8_t* valid, double* acc,
                              cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  column_sum_kernel<<<(dim + 31) / 32, 256, 0, stream>>>(v, rows, dim, valid, acc);
  return cudaGetLastError();
}

cudaError_t center_launch(const double* acc, int32_t dim, int64_t used, float* center, cudaStream_t stream) {
  center_kernel<<<(dim + 127) / 128, 128, 0, stream>>>(acc, dim, used, center);
  return cudaGetLastError();
}

cudaError_t pack_rows_launch(const float* v, int64_t rows, int32_t dim, const float* center, const uint8_t* valid,
                             int32_t wpad, uint64_t* bits, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const unsigned grid = (unsigned)((rows + kRowWarps - 1) / kRowWarps);
  pack_rows_kernel<<<grid, kRowWarps * 32, 0, stream>>>(v, rows, dim, center, valid, wpad, bits);
  return cudaGetLastError();
}

}  // namespace fi8
