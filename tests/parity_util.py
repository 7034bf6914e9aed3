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
