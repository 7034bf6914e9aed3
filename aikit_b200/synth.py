"""Seeded synthetic corpora (ctypes over lib/libfi8_synth.so).

Stand-ins for the benchmark configurations' data (the reference's Model2Vec
embeddings are not available here). See csrc/synth.c for the exact recipe;
every value is a pure function of (seed, stream, row, column).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libfi8_synth.so")

UNIT, MIXTURE, TIES = 0, 1, 2
# stream ids
CORPUS, QUERIES, CENTERS = 1, 2, 3

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from .build import build_synth
            build_synth()
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        L.syn_rows.argtypes = [C.c_int, C.c_uint64, C.c_uint64, P, C.c_int64, C.c_float, C.c_int64,
                               C.c_int64, C.c_int64, P, P, P, C.c_int]
        L.syn_normal_rows.argtypes = [C.c_uint64, C.c_uint64, C.c_int64, C.c_int64, C.c_int64, P]
        L.syn_column_sums.argtypes = [C.c_int, C.c_uint64, C.c_uint64, P, C.c_int64, C.c_float, C.c_int64,
                                      C.c_int64, C.c_int64, P, C.c_int]
        L.syn_binary_rows.argtypes = [C.c_int, C.c_uint64, C.c_uint64, P, C.c_int64, C.c_float, C.c_int64,
                                      C.c_int64, C.c_int64, P, P, P, P, C.c_int]
        L.syn_quantize_row.restype = C.c_float
        L.syn_quantize_row.argtypes = [P, C.c_int64, P, C.c_float]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _threads(nthreads: int) -> int:
    return nthreads or (os.cpu_count() or 1)


def centers(seed: int, ncl: int, d: int) -> np.ndarray:
    out = np.empty((ncl, d), np.float32)
    lib().syn_normal_rows(seed, CENTERS, 0, ncl, d, _p(out))
    return out


class Recipe:
    """One synthetic distribution: kind UNIT, MIXTURE (ncl, sigma) or TIES."""

    def __init__(self, kind: int, d: int, seed: int = 1, ncl: int = 0, sigma: float = 0.0):
        self.kind, self.d, self.seed, self.ncl, self.sigma = kind, d, seed, ncl, sigma
        self._centers = centers(seed, ncl, d) if kind == MIXTURE else None

    def _call(self, stream, row0, n, out_f, out_q, out_s, nthreads):
        lib().syn_rows(self.kind, self.seed, stream, _p(self._centers), self.ncl, self.sigma,
                       row0, n, self.d, _p(out_f), _p(out_q), _p(out_s), _threads(nthreads))

    def floats(self, n: int, row0: int = 0, stream: int = CORPUS, nthreads: int = 0) -> np.ndarray:
        out = np.empty((n, self.d), np.float32)
        self._call(stream, row0, n, out, None, None, nthreads)
        return out

    def codes(self, n: int, row0: int = 0, stream: int = CORPUS, nthreads: int = 0, out_q=None, out_s=None):
        """Corpus rows quantized as NewFlatI8 does (or the fixed-scale ties codes)."""
        q = out_q if out_q is not None else np.empty((n, self.d), np.int8)
        s = out_s if out_s is not None else np.empty(n, np.float32)
        self._call(stream, row0, n, None, q, s, nthreads)
        return q, s

    def center(self, n: int, row0: int = 0, nthreads: int = 0) -> np.ndarray:
        """float32(column mean) of rows [row0, row0+n), accumulated in float64
        (the centring of newBinaryPrefilter, ann/flat_binary_prefilter.go:64-85,
        summed block-wise so it can be generated in parallel)."""
        acc = np.empty(self.d, np.float64)
        lib().syn_column_sums(self.kind, self.seed, CORPUS, _p(self._centers), self.ncl, self.sigma,
                              row0, n, self.d, _p(acc), _threads(nthreads))
        return (acc / float(n)).astype(np.float32)

    def binary(self, n: int, center=None, row0: int = 0, nthreads: int = 0, with_codes: bool = True):
        """A FlatBinaryI8 corpus without materialising float rows: packed sign
        codes [n, ceil(d/64)] uint64 of (v - center), and the int8 rows and
        scales (None when with_codes is False)."""
        words = (self.d + 63) // 64
        bits = np.empty((n, words), np.uint64)
        q = np.empty((n, self.d), np.int8) if with_codes else None
        s = np.empty(n, np.float32) if with_codes else None
        ctr = None if center is None else np.ascontiguousarray(center, np.float32)
        lib().syn_binary_rows(self.kind, self.seed, CORPUS, _p(self._centers), self.ncl, self.sigma, row0, n,
                              self.d, _p(ctr), _p(bits), _p(q), _p(s), _threads(nthreads))
        return bits, q, s

    def queries(self, m: int, row0: int = 0, nthreads: int = 0) -> np.ndarray:
        return self.floats(m, row0=row0, stream=QUERIES, nthreads=nthreads)


def quantize_row(row, zero_scale: float = 1.0):
    row = np.ascontiguousarray(row, np.float32)
    q = np.empty(row.shape[0], np.int8)
    s = lib().syn_quantize_row(_p(row), row.shape[0], _p(q), zero_scale)
    return q, np.float32(s)
