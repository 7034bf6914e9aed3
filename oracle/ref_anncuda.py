"""The reference's own device path, for comparison on the same B200. TEST
INFRASTRUCTURE.

``oracle/_ref/libref_anncuda.so`` holds the kernels of the reference's
gpu/anncuda/gemv_w8a8.cu, compiled for sm_100a from the reference source tree
(``make -C oracle ref``), behind ``oracle/ref_anncuda.cu``: a launcher that
restates the host-side choices of gpu/anncuda/backend.go (launchBatch :675-712,
launchTopK :468-510). Only tests, the parity-fixture generator and the
benchmark's comparator leg use it; the product never loads it.

All pointers are device pointers (e.g. torch tensors' data_ptr()); the
queries are int8 rows quantized on the host as the reference's
quantizeRowInt8 does (backend.go:270-298; ``oracle.quantize_queries``).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libref_anncuda.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with `make -C oracle ref` where the "
                                    "reference source tree is present")
        L = C.CDLL(LIB_PATH)
        P, U32 = C.c_void_p, C.c_uint32
        L.ref_plan_create.argtypes = [U32, U32, U32, U32, C.c_int, P]
        L.ref_plan_destroy.argtypes = [P]
        L.ref_score_launch.argtypes = [P, P, P, P, P, P, P]
        L.ref_topk_launch.argtypes = [P, P, P, P, P]
        L.ref_plan_launches.argtypes = [P]
        _lib = L
    return _lib


class RefTopK:
    """One TopKBatch shape (n rows of dim, M queries, k) on the current device:
    ``score`` is launchBatch (M x n f32 scores), ``topk`` is launchTopK over
    those scores (consumed by the k-pass kernel), both stream-ordered."""

    def __init__(self, n: int, dim: int, M: int, k: int, sm_count: int):
        self._p = C.c_void_p()
        rc = lib().ref_plan_create(n, dim, M, k, sm_count, C.byref(self._p))
        if rc != 0:
            raise RuntimeError(f"ref_plan_create failed ({rc})")
        self.launches = lib().ref_plan_launches(self._p)

    def score(self, codes: int, scales: int, qi8: int, qscale: int, scores: int, stream: int = 0) -> None:
        if lib().ref_score_launch(self._p, codes, scales, qi8, qscale, scores, stream) != 0:
            raise RuntimeError("reference scoring launch failed")

    def topk(self, scores: int, idx: int, val: int, stream: int = 0) -> None:
        if lib().ref_topk_launch(self._p, scores, idx, val, stream) != 0:
            raise RuntimeError("reference top-k launch failed")

    def close(self) -> None:
        if self._p:
            lib().ref_plan_destroy(self._p)
            self._p = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
