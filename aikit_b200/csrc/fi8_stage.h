// fi8_stage.h -- host-to-device uploads through a pinned double buffer.
//
// A corpus arrives in pageable host memory (a Go slice, a numpy array, or an
// mmap of an FI8 file whose pages come from the page cache,
// ann/flat_i8_mmap.go:33-212). A plain cudaMemcpy from pageable memory stages
// through a small driver buffer at a fraction of the link rate. Here host
// threads copy rows into one of two pinned buffers while the DMA engine
// drains the other, and rows can be re-pitched on the way (the device rows
// are padded to 16 bytes; padding bytes are written as zero).
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace fi8 {

class PinnedStager {
 public:
  static constexpr size_t kBufBytes = (size_t)64 << 20;

  PinnedStager() = default;
  PinnedStager(const PinnedStager&) = delete;
  PinnedStager& operator=(const PinnedStager&) = delete;
  ~PinnedStager() { release(); }

  cudaError_t init() {
    for (int b = 0; b < 2; b++) {
      cudaError_t e = cudaMallocHost(reinterpret_cast<void**>(&pin_[b]), kBufBytes);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev_[b], cudaEventDisableTiming);
      if (e != cudaSuccess) return e;
    }
    const unsigned hw = std::thread::hardware_concurrency();
    threads_ = (int)std::max(1u, std::min(hw ? hw : 1u, 16u));
    return cudaSuccess;
  }

  // rows rows of src_w bytes, src_pitch apart -> device rows dst_pitch apart
  // (dst_pitch >= src_w; the bytes past src_w are zero). Stream-ordered on st;
  // the host data may be reused once finish() returns.
  cudaError_t put_rows(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t src_w, int64_t rows,
                       cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    const int64_t per = std::max<int64_t>(1, (int64_t)(kBufBytes / dst_pitch));
    if ((size_t)per * dst_pitch > kBufBytes) return cudaErrorInvalidValue;  // a row larger than a buffer
    const unsigned char* s = static_cast<const unsigned char*>(src);
    unsigned char* d = static_cast<unsigned char*>(dst);
    for (int64_t r0 = 0; r0 < rows; r0 += per) {
      const int64_t nr = std::min(per, rows - r0);
      const int b = next_;
      if (used_[b]) {
        cudaError_t e = cudaEventSynchronize(ev_[b]);  // its previous DMA is done
        if (e != cudaSuccess) return e;
      }
      fill(pin_[b], dst_pitch, s + (size_t)r0 * src_pitch, src_pitch, src_w, nr);
      cudaError_t e = cudaMemcpyAsync(d + (size_t)r0 * dst_pitch, pin_[b], (size_t)nr * dst_pitch,
                                      cudaMemcpyHostToDevice, st);
      if (e == cudaSuccess) e = cudaEventRecord(ev_[b], st);
      if (e != cudaSuccess) return e;
      used_[b] = true;
      next_ ^= 1;
    }
    return cudaSuccess;
  }

  // Wait until both buffers are free (their copies have completed).
  cudaError_t finish() {
    for (int b = 0; b < 2; b++)
      if (used_[b]) {
        cudaError_t e = cudaEventSynchronize(ev_[b]);
        if (e != cudaSuccess) return e;
        used_[b] = false;
      }
    return cudaSuccess;
  }

  void release() {
    finish();
    for (int b = 0; b < 2; b++) {
      if (pin_[b]) cudaFreeHost(pin_[b]);
      if (ev_[b]) cudaEventDestroy(ev_[b]);
      pin_[b] = nullptr;
      ev_[b] = nullptr;
    }
  }

 private:
  // Copy rows into the pinned buffer, split over host threads by rows.
  void fill(unsigned char* out, size_t dst_pitch, const unsigned char* src, size_t src_pitch, size_t src_w,
            int64_t rows) const {
    auto part = [=](int64_t a, int64_t b) {
      if (dst_pitch == src_w && src_pitch == src_w) {
        std::memcpy(out + (size_t)a * dst_pitch, src + (size_t)a * src_pitch, (size_t)(b - a) * src_w);
        return;
      }
      for (int64_t r = a; r < b; r++) {
        std::memcpy(out + (size_t)r * dst_pitch, src + (size_t)r * src_pitch, src_w);
        if (dst_pitch > src_w) std::memset(out + (size_t)r * dst_pitch + src_w, 0, dst_pitch - src_w);
      }
    };
    const size_t bytes = (size_t)rows * dst_pitch;
    const int t = (int)std::min<int64_t>(threads_, std::max<int64_t>(1, (int64_t)(bytes >> 22)));  // >= 4 MB each
    if (t <= 1) {
      part(0, rows);
      return;
    }
    std::vector<std::thread> pool;
    pool.reserve(t);
    for (int i = 0; i < t; i++) pool.emplace_back(part, rows * i / t, rows * (i + 1) / t);
    for (auto& th : pool) th.join();
  }

  unsigned char* pin_[2] = {nullptr, nullptr};
  cudaEvent_t ev_[2] = {nullptr, nullptr};
  bool used_[2] = {false, false};
  int next_ = 0;
  int threads_ = 1;
};

}  // namespace fi8
