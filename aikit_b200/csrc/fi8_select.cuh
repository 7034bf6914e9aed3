// fi8_select.cuh -- exact top-K building blocks shared by the scan, GEMM and
// select kernels: warp-aggregated appends into a shared candidate buffer, a
// bitonic sort/compaction run by one 256-thread group (named barrier), and the
// "top-k of two sorted lists" tree merge.
//
// Keys are the packed (score desc, index asc) uint64 of fi8_device.cuh, so
// every operation here is a selection of the largest distinct integers.
#pragma once

#include "fi8_device.cuh"

namespace fi8 {

constexpr int kGroupThreads = 256;

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ int next_pow2_dev(int x) {
  int p = 2;
  while (p < x) p <<= 1;
  return p;
}

// Append `key` (when take) to buf using one shared atomic per warp.
__device__ __forceinline__ void warp_append(bool take, uint64_t key, uint64_t* buf, int* s_count) {
  const uint32_t mask = __ballot_sync(0xffffffffu, take);
  if (mask == 0) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(mask) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(s_count, __popc(mask));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (take) buf[base + __popc(mask & lanemask_lt())] = key;
}

// Bitonic sort (descending) of n = 2^j keys by a group of NT threads that
// synchronize on named barrier `bar`.
template <int NT = kGroupThreads>
__device__ inline void group_sort_desc(uint64_t* buf, int n, int gtid, int bar) {
  const int half = n >> 1;
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = gtid; i < half; i += NT) {
        const int lo = 2 * stride * (i / stride) + (i % stride);
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t a = buf[lo], b = buf[hi];
        if ((a < b) == desc) {
          buf[lo] = b;
          buf[hi] = a;
        }
      }
      named_sync(bar, NT);
    }
  }
}

// Sort the first cnt keys, keep the best k, raise (and optionally publish) the
// group threshold. All NT threads of the group call it with the same cnt.
template <int NT = kGroupThreads>
__device__ inline void group_compact(uint64_t* buf, int cnt, int k, int* s_count, unsigned long long* s_local_thr,
                                     unsigned long long* gthr, int gtid, int bar) {
  const int n2 = next_pow2_dev(cnt < 2 ? 2 : cnt);
  for (int i = cnt + gtid; i < n2; i += NT) buf[i] = kEmptyKey;
  named_sync(bar, NT);
  group_sort_desc<NT>(buf, n2, gtid, bar);
  if (gtid == 0) {
    *s_count = cnt < k ? cnt : k;
    if (cnt >= k) {
      const unsigned long long t = buf[k - 1];
      if (t > *s_local_thr) *s_local_thr = t;
      if (gthr) atomicMax(gthr, t);
    }
  }
  named_sync(bar, NT);
}

// Tree-merge `total` sorted (descending) lists of kp keys held in slots
// [0, total) into slot 0. Each pairwise step keeps the top kp of two sorted
// lists: c[i] = max(a[i], b[kp-1-i]) is bitonic and holds exactly that top kp,
// and a bitonic merge sorts it. All pairs of a level advance together.
__device__ inline void tree_merge_slots(uint64_t* slots, int total, int kp, int gtid, int bar) {
  for (int step = 1; step < total; step <<= 1) {
    const int npairs = (total - step + 2 * step - 1) / (2 * step);
    for (int w = gtid; w < npairs * kp; w += kGroupThreads) {
      const int j = (w / kp) * 2 * step, i = w % kp;
      const uint64_t a = slots[(size_t)j * kp + i];
      const uint64_t b = slots[(size_t)(j + step) * kp + (kp - 1 - i)];
      slots[(size_t)j * kp + i] = a > b ? a : b;
    }
    named_sync(bar, kGroupThreads);
    for (int stride = kp >> 1; stride > 0; stride >>= 1) {
      for (int w = gtid; w < npairs * (kp >> 1); w += kGroupThreads) {
        const int j = (w / (kp >> 1)) * 2 * step, i = w % (kp >> 1);
        uint64_t* s = slots + (size_t)j * kp;
        const int lo = 2 * stride * (i / stride) + (i % stride);
        const int hi = lo + stride;
        const uint64_t a = s[lo], b = s[hi];
        if (a < b) {
          s[lo] = b;
          s[hi] = a;
        }
      }
      named_sync(bar, kGroupThreads);
    }
  }
}

// Top kp of m global lists (each `len` <= kp keys, stride `stride` keys apart,
// sorted descending, 0 = empty) into slots[0..kp). Uses as many shared slots
// as fit; slot 0 carries the running result between rounds.
__device__ inline void merge_global_lists(const uint64_t* lists, int m, int len, size_t stride, int kp,
                                          uint64_t* slots, int nslots, int gtid, int bar) {
  int done = 0;
  bool have = false;
  if (m == 0) {
    for (int i = gtid; i < kp; i += kGroupThreads) slots[i] = kEmptyKey;
    named_sync(bar, kGroupThreads);
    return;
  }
  while (done < m) {
    const int base = have ? 1 : 0;
    const int c = min(nslots - base, m - done);
    for (int w = gtid; w < c * kp; w += kGroupThreads) {
      const int l = w / kp, i = w % kp;
      slots[(size_t)(base + l) * kp + i] = i < len ? __ldcg(lists + (size_t)(done + l) * stride + i) : kEmptyKey;
    }
    named_sync(bar, kGroupThreads);
    tree_merge_slots(slots, base + c, kp, gtid, bar);
    done += c;
    have = true;
  }
}

}  // namespace fi8
