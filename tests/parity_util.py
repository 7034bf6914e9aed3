"""Shared parity helpers for the GPU tests (oracle side = the CPU checker)."""
import numpy as np

import oracle


def oracle_topk(bq, bs, Q, k):
    """FlatI8.Query (ann/flat_i8.go:124) per query on the CPU oracle, padded
    to k with index -1 like the device answer."""
    idx = np.full((len(Q), k), -1, np.int64)
    sc = np.zeros((len(Q), k), np.float32)
    for m, q in enumerate(Q):
        i, s = oracle.flat_i8_query(bq, bs, q, k)
        idx[m, :len(i)] = i
        sc[m, :len(s)] = np.asarray(s, np.float32)
    return idx, sc


def assert_same(gidx, gsc, widx, wsc, what=""):
    """Identical indices and bit-identical float32 scores."""
    assert gidx.shape == widx.shape, what
    bad = np.nonzero(gidx != widx)
    assert bad[0].size == 0, f"{what}: first index mismatch at {bad[0][0]},{bad[1][0]}: " \
        f"gpu {gidx[bad[0][0]]} vs oracle {widx[bad[0][0]]}"
    valid = widx >= 0
    assert gsc[valid].tobytes() == wsc[valid].tobytes(), f"{what}: scores differ"


def make_keys(idx, score):
    """The library's packed ranking key (score desc, index asc) on the host:
    order-preserving image of the float32 score (-0 == +0) in bits 63..32,
    0x7FFFFFFF - index in bits 31..1, bit 0 set for a -0.0 score; 0 = empty
    (index < 0)."""
    idx = np.asarray(idx, np.int64)
    b = np.asarray(score, np.float32).view(np.uint32).astype(np.uint64)
    negzero = (b == 0x80000000).astype(np.uint64)
    b = np.where(negzero == 1, np.uint64(0), b)
    ord_ = np.where(b & np.uint64(0x80000000), ~b & np.uint64(0xFFFFFFFF), b | np.uint64(0x80000000))
    key = (ord_ << np.uint64(32)) | (((np.uint64(0x7FFFFFFF) - idx.astype(np.uint64)) & np.uint64(0x7FFFFFFF))
                                     << np.uint64(1)) | negzero
    return np.where(idx < 0, np.uint64(0), key)


def top_keys(keys, k):
    """Top k of a key array (descending), 0-padded."""
    keys = np.sort(np.asarray(keys, np.uint64).reshape(-1))[::-1][:k]
    out = np.zeros(k, np.uint64)
    out[:len(keys)] = keys
    return out
