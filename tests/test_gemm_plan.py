"""The batched path's row-range plan (fi8_gemm_plan, a host-only C-ABI call):
the ranges a TopKBatch of M queries at k over n rows runs as, one GEMM launch
and one select each. CPU only.

The plan's rules, restated here to pin them:
  * the first range takes max(k, 4096) rows (rounded up to 256-row tiles);
  * then each range ends at F times its start, rounded up to a 256-row tile;
    batches of up to 64 queries grow by 16 below 16K rows and 64 above, larger
    batches by 8 (2 when k >= 512); every factor is capped by the per-query
    candidate buffer, room = cap / (4k) with cap = 8K..64K keys (256 MB of keys
    across the batch at most);
  * a short tail (under half the range before it) joins that range when the
    joined range still fits the buffer's growth room.
Exactness never depends on the plan (every range is filtered against the k-th
best key of the rows before it); the plan only sets how many candidates each
range admits and how many launches a batch takes.
"""
import ctypes as C

import numpy as np
import pytest

from aikit_b200 import Fi8Error
from aikit_b200._ffi import FI8_ERR_ARG, check, lib


def device_plan(n, M, k, max_bounds=64):
    out = np.zeros(max_bounds, np.int64)
    cnt = C.c_int32(0)
    check(lib().fi8_gemm_plan(n, M, k, out.ctypes.data, max_bounds, C.byref(cnt)))
    return out[:cnt.value + 1].tolist()


def pow2_ge(x):
    p = 1
    while p < x:
        p <<= 1
    return p


def restated_plan(n, M, k):
    cap = min(pow2_ge(max(8192, min(65536, (1 << 25) // M))), 65536)
    room = max(4, cap // (4 * k))
    fine = M > 64
    f1 = min((2 if k >= 512 else 8) if fine else 16, room)
    f2 = f1 if fine else min(64, room)
    hi = -(-max(k, 4096) // 256) * 256
    lo, bounds = 0, [0]
    while lo < n:
        h = min(n, hi)
        if lo > 0 and h < n and n - h < (h - lo) // 2 and n - lo <= lo * room:
            h = n
        bounds.append(h)
        lo = h
        f = f2 if lo >= 16 * 1024 else f1
        hi = -(-(lo * f) // 256) * 256
    return bounds


def test_plans_of_the_profiled_launches():
    K = 1024
    # W8A8 batch 4096 at k = 100 over 1M rows: growth 8
    assert device_plan(1_000_000, 4096, 100) == [0, 4096, 32768, 262144, 1_000_000]
    # the Hamming prefilter's batch 512 at cand = 1000 over 1M rows: growth 2
    assert device_plan(1_000_000, 512, 1000) == [0, 4096, 8192, 16384, 32768, 65536, 131072, 262144, 524288,
                                                  1_000_000]
    # C5: batch 1024 at k = 1000 over 16M rows (the profiled shape)
    assert device_plan(16_000_000, 1024, 1000) == [0] + [4096 << i for i in range(12)] + [16_000_000]
    # C2: batch 64 at k = 100 over 10M rows: growth 16, then 64
    assert device_plan(10_000_000, 64, 100) == [0, 4096, 65536, 4 * K * K, 10_000_000]
    # a row shard of C2 over 8 GPUs
    assert device_plan(1_250_000, 64, 100) == [0, 4096, 65536, 1_250_000]


def test_plan_equals_the_restated_rules():
    rng = np.random.default_rng(7)
    cases = [(1, 1, 1), (4096, 2, 100), (4097, 2, 100), (256, 300, 255), (50_000_000, 4096, 100),
             (200_000_000, 1, 10), (25_000_000, 512, 1000), (2_147_000_000, 8, 4096)]
    for _ in range(3000):
        n = int(rng.integers(1, 1 << int(rng.integers(1, 31))))
        M = int(rng.choice([1, 2, 3, 16, 63, 64, 65, 128, 200, 512, 1024, 4096, 20000]))
        k = int(rng.choice([1, 5, 10, 100, 511, 512, 1000, 2048, 4096]))
        cases.append((n, M, k))
    for n, M, k in cases:
        assert device_plan(n, M, k) == restated_plan(n, M, k), (n, M, k)


@pytest.mark.parametrize("M", [1, 64, 65, 4096])
@pytest.mark.parametrize("k", [1, 100, 1000, 4096])
def test_plan_properties(M, k):
    for n in (1, 255, 256, 4095, 4096, 4097, 16_384, 100_003, 10_000_000, 2_000_000_000):
        b = device_plan(n, M, k)
        assert b[0] == 0 and b[-1] == n
        assert all(x < y for x, y in zip(b, b[1:]))
        assert all(x % 256 == 0 for x in b[1:-1])  # whole 256-row GEMM tiles
        assert b[1] == min(n, -(-max(k, 4096) // 256) * 256) or len(b) == 2
        # launches per batch stay few at any size: growth 2 (k >= 512) reaches
        # 2e9 rows in 20 ranges, the others in at most 12
        assert len(b) - 1 <= (20 if k >= 512 and M > 64 else 12)


def test_plan_rejects_bad_arguments():
    out = np.zeros(4, np.int64)
    cnt = C.c_int32(-1)
    for n, M, k in ((0, 1, 1), (10, 0, 1), (10, 1, 0), (-5, 2, 2)):
        with pytest.raises(Fi8Error):
            check(lib().fi8_gemm_plan(n, M, k, out.ctypes.data, 4, C.byref(cnt)))
    # too small an output: the error carries the range count
    rc = lib().fi8_gemm_plan(10_000_000, 64, 100, out.ctypes.data, 3, C.byref(cnt))
    assert rc == FI8_ERR_ARG and cnt.value == 4
