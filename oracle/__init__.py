"""CPU oracle for the FlatI8 / FlatBinaryI8 exact-scan path. TEST INFRASTRUCTURE.

A ctypes view of ``oracle/lib/libfi8_oracle.so``, the C restatement of the
reference's Go path (github.com/townsendmerino/aikit). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
module, and only as the checker: the product (``aikit_b200``) never calls it and
has no CPU fallback.

Each wrapper names the reference file:line it restates; the C source carries
the line-level citations. Parity pinning status: pinned by the reference's
literal test vectors and known-answer relations plus its real-data fixtures,
and by outputs of the reference's own CUDA kernels (gpu/anncuda/gemv_w8a8.cu
compiled for sm_100a, ``oracle/ref_anncuda.py``) run on a B200: W8A8 scores
and top-k ids and scores, committed as ``tests/golden/ref_anncuda_outputs.npz``.
The Go path itself cannot run (no Go toolchain here or on the GPU box).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "lib", "libfi8_oracle.so")
_lib = None

_P = C.c_void_p
_I64 = C.c_int64


REFERENCE = "/root/reference"


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off), and,
    where the reference source tree is present (the build machine, not the GPU
    box, which only receives the built files), the reference's own CUDA
    kernels into oracle/_ref/ (see ref_anncuda.py)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    if os.path.isfile(os.path.join(REFERENCE, "gpu", "anncuda", "gemv_w8a8.cu")):
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF={REFERENCE}"], check=True)
    return _LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.or_quantize_row.restype = C.c_float
        L.or_quantize_row.argtypes = [_P, _I64, _P, C.c_float]
        L.or_quantize_rows.argtypes = [_P, _I64, _I64, _P, _P, C.c_float]
        L.or_dot_i8_scalar.restype = C.c_int32
        L.or_dot_i8_scalar.argtypes = [_P, _P, _I64]
        L.or_dot_i8.restype = C.c_int32
        L.or_dot_i8.argtypes = [_P, _P, _I64]
        L.or_w8a8.argtypes = [_P, _P, _I64, _P, _P, _I64, _I64, _P, C.c_int]
        L.or_top_hits.restype = _I64
        L.or_top_hits.argtypes = [_P, _I64, _I64, _P, _P, _P]
        L.or_flat_i8_query.restype = _I64
        L.or_flat_i8_query.argtypes = [_P, _P, _I64, _I64, _P, _I64, _P, _P, _P, C.c_int]
        L.or_merge_hits.restype = _I64
        L.or_merge_hits.argtypes = [_P, _P, _I64, _I64, _P, _P]
        L.or_center.restype = _I64
        L.or_center.argtypes = [_P, _I64, _I64, _P, _P]
        L.or_pack_row.argtypes = [_P, _P, _I64, _P]
        L.or_pack_codes.argtypes = [_P, _P, _I64, _I64, _P, _P]
        L.or_hamming_rows.argtypes = [_P, _P, _I64, _I64, _P]
        L.or_prefilter_hist.restype = _I64
        L.or_prefilter_hist.argtypes = [_P, _P, _I64, _I64, _I64, _P]
        L.or_prefilter_heap.restype = _I64
        L.or_prefilter_heap.argtypes = [_P, _P, _I64, _I64, _I64, _P, C.c_int, _P]
        L.or_flat_binary_i8_query.restype = _I64
        L.or_flat_binary_i8_query.argtypes = [_P, _P, _I64, _P, _P, _I64, _I64, _I64,
                                              _P, _I64, _P, _P, _P, C.c_int]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def nthreads_default() -> int:
    return os.cpu_count() or 1


# --- quantization: linalg/quant.go:43-71, :83, :171 --------------------------

def quantize_row(row, zero_scale: float):
    row = _c(row, np.float32)
    q = np.empty(row.shape[0], np.int8)
    s = lib().or_quantize_row(_ptr(row), row.shape[0], _ptr(q), zero_scale)
    return q, np.float32(s)


def quantize_rows(v, zero_scale: float = 1.0):
    """QuantizeRowsInt8 (linalg/quant.go:21-31): corpus rows, all-zero -> 1."""
    v = _c(v, np.float32)
    n, d = v.shape
    q = np.empty((n, d), np.int8)
    s = np.empty(n, np.float32)
    lib().or_quantize_rows(_ptr(v), n, d, _ptr(q), _ptr(s), zero_scale)
    return q, s


def quantize_queries(v):
    """quantizeRowInt8 (linalg/quant.go:171): activation rows, all-zero -> 0."""
    return quantize_rows(v, 0.0)


# --- dot / W8A8: linalg/quant.go:150, quant_i8_amd64.go:10, quant.go:248 -----

def dot_i8(a, b, scalar: bool = False) -> int:
    a = _c(a, np.int8)
    b = _c(b, np.int8)
    f = lib().or_dot_i8_scalar if scalar else lib().or_dot_i8
    return int(f(_ptr(a), _ptr(b), a.shape[0]))


def w8a8(aq, ascales, bq, bscales, nthreads: int = 0):
    aq = _c(np.atleast_2d(aq), np.int8)
    ascales = _c(np.atleast_1d(ascales), np.float32)
    bq = _c(bq, np.int8)
    bscales = _c(bscales, np.float32)
    M, d = aq.shape
    N = bq.shape[0]
    dst = np.empty((M, N), np.float32)
    lib().or_w8a8(_ptr(aq), _ptr(ascales), M, _ptr(bq), _ptr(bscales), N, d,
                  _ptr(dst), nthreads or nthreads_default())
    return dst


# --- selection: ann/flat_i8.go:214-246, topk/topk.go, ann/backend.go:262 ----

def top_hits(scores, k: int, keep=None):
    scores = _c(scores, np.float32)
    n = scores.shape[0]
    cap = max(n, 1)
    idx = np.empty(cap, np.int64)
    sc = np.empty(cap, np.float64)
    keep = None if keep is None else _c(keep, np.uint8)
    c = lib().or_top_hits(_ptr(scores), n, k, _ptr(keep), _ptr(idx), _ptr(sc))
    return idx[:c].copy(), sc[:c].copy()


def flat_i8_query(bq, scales, q, k: int, keep=None, nthreads: int = 0):
    """FlatI8.Query / QueryFilter CPU path (ann/flat_i8.go:124-206).

    Returns (idx int64[], score float64[]) or None for the reference's nil.
    """
    bq = _c(bq, np.int8)
    scales = _c(scales, np.float32)
    n = bq.shape[0]
    d = bq.shape[1] if bq.ndim == 2 else 0
    q = _c(q, np.float32)
    if n == 0 or q.shape[0] != d:
        return None
    cap = max(n, 1)
    idx = np.empty(cap, np.int64)
    sc = np.empty(cap, np.float64)
    keep = None if keep is None else _c(keep, np.uint8)
    c = lib().or_flat_i8_query(_ptr(bq), _ptr(scales), n, d, _ptr(q), k, _ptr(keep),
                               _ptr(idx), _ptr(sc), nthreads or nthreads_default())
    if c < 0:
        return None
    return idx[:c].copy(), sc[:c].copy()


def merge_hits(parts, k: int):
    """queryBatchSharded's merge (ann/backend.go:262-277)."""
    idx = np.concatenate([np.asarray(p[0], np.int64) for p in parts]) if parts else np.empty(0, np.int64)
    sc = np.concatenate([np.asarray(p[1], np.float64) for p in parts]) if parts else np.empty(0, np.float64)
    idx = _c(idx, np.int64)
    sc = _c(sc, np.float64)
    cap = max(idx.shape[0], 1)
    oi = np.empty(cap, np.int64)
    os_ = np.empty(cap, np.float64)
    c = lib().or_merge_hits(_ptr(idx), _ptr(sc), idx.shape[0], k, _ptr(oi), _ptr(os_))
    return oi[:c].copy(), os_[:c].copy()


# --- binary prefilter: ann/flat_binary_prefilter.go, linalg/hamming.go -------

def packed_words(dim: int) -> int:
    return (dim + 63) // 64


def center(v, valid=None):
    """Returns the float32 corpus mean, or None when no row is valid."""
    v = _c(v, np.float32)
    n, d = v.shape
    c = np.empty(d, np.float32)
    valid = None if valid is None else _c(valid, np.uint8)
    used = lib().or_center(_ptr(v), n, d, _ptr(valid), _ptr(c))
    return c if used > 0 else None


def pack_row(v, ctr=None):
    v = _c(v, np.float32)
    d = v.shape[0]
    out = np.empty(packed_words(d), np.uint64)
    ctr = None if ctr is None else _c(ctr, np.float32)
    lib().or_pack_row(_ptr(v), _ptr(ctr), d, _ptr(out))
    return out


def pack_codes(v, ctr=None, valid=None):
    v = _c(v, np.float32)
    n, d = v.shape
    out = np.empty((n, packed_words(d)), np.uint64)
    ctr = None if ctr is None else _c(ctr, np.float32)
    valid = None if valid is None else _c(valid, np.uint8)
    lib().or_pack_codes(_ptr(v), _ptr(ctr), n, d, _ptr(valid), _ptr(out))
    return out


def hamming_rows(qc, codes):
    qc = _c(qc, np.uint64)
    codes = _c(codes, np.uint64)
    n, w = codes.shape
    out = np.empty(n, np.uint16)
    lib().or_hamming_rows(_ptr(qc), _ptr(codes), w, n, _ptr(out))
    return out


def prefilter_hist(qc, codes, dim: int, cand: int):
    qc = _c(qc, np.uint64)
    codes = _c(codes, np.uint64)
    n = codes.shape[0]
    ids = np.empty(max(cand, 1), np.int32)
    c = lib().or_prefilter_hist(_ptr(qc), _ptr(codes), n, dim, cand, _ptr(ids))
    return ids[:c].copy()


def prefilter_heap(qc, codes, dim: int, cand: int, keep=None, nshards: int = 1):
    qc = _c(qc, np.uint64)
    codes = _c(codes, np.uint64)
    n = codes.shape[0]
    ids = np.empty(max(cand, 1), np.int32)
    keep = None if keep is None else _c(keep, np.uint8)
    c = lib().or_prefilter_heap(_ptr(qc), _ptr(codes), n, dim, cand, _ptr(keep), nshards, _ptr(ids))
    return ids[:c].copy()


def flat_binary_i8_query(codes, ctr, bq, scales, over: int, q, k: int, keep=None,
                         nthreads: int = 0):
    """FlatBinaryI8.Query / QueryFilter (ann/flat_binary_i8.go:86-153)."""
    codes = _c(codes, np.uint64)
    bq = _c(bq, np.int8)
    scales = _c(scales, np.float32)
    q = _c(q, np.float32)
    n, d = bq.shape
    if n == 0 or q.shape[0] != d:
        return None
    ctr = None if ctr is None else _c(ctr, np.float32)
    cap = max(n, 1)
    idx = np.empty(cap, np.int64)
    sc = np.empty(cap, np.float64)
    keep = None if keep is None else _c(keep, np.uint8)
    c = lib().or_flat_binary_i8_query(_ptr(codes), _ptr(ctr), codes.shape[1], _ptr(bq),
                                      _ptr(scales), n, d, over, _ptr(q), k, _ptr(keep),
                                      _ptr(idx), _ptr(sc), nthreads or nthreads_default())
    if c < 0:
        return None
    return idx[:c].copy(), sc[:c].copy()
