"""Parity at BASELINE.json's full sizes: the C3 headline, C2, C5 and C4's
per-GPU FlatBinaryI8 shard.

The other GPU tests check the device paths against the oracle at sizes the
oracle finishes in a second or two. These run the configurations `bench.py`
measures at their full size, where the range plan runs all its ranges, the
candidate buffers and the GEMM's persistent grid carry their real load, and
the int32 dot products and float32 scores cover the whole corpus. A full
batch runs on the device through the host API; two sampled queries of that
batch (its first and its last) are checked against the oracle's full scan,
run chunk by chunk as the corpus is generated. Selection decomposes, so the
chunk answers merge exactly by queryBatchSharded's rule
(ann/backend.go:262-277). The C3 test holds 51 GB on the device and takes
about 25 s on a B200 (most of it generating the corpus); C5 holds 26 GB and
takes about 6 s, C2 8 GB and a few seconds, C4's shard about 55 GB (codes,
int8 rows and the tensor prefilter's sign rows) and about 25 s.
"""
import os

import numpy as np
import pytest

import oracle
from aikit_b200 import synth

from parity_util import assert_same

pytestmark = pytest.mark.gpu

CHUNK = 1 << 20  # rows generated, checked and uploaded at a time


def _build_with_oracle(backend, recipe, n, d, samples, k):
    """Upload n rows of the recipe block by block; the oracle answers the
    sampled queries over every block as it goes. Returns the index and, per
    sampled query, the oracle's (ids, float32 scores) padded to k."""
    threads = os.cpu_count() or 1
    ix = backend.NewI8IndexEmpty(n, d)
    q = np.empty((CHUNK, d), np.int8)
    s = np.empty(CHUNK, np.float32)
    best = [(np.empty(0, np.int64), np.empty(0, np.float64)) for _ in samples]
    for r0 in range(0, n, CHUNK):
        m = min(CHUNK, n - r0)
        recipe.codes(m, row0=r0, out_q=q[:m], out_s=s[:m])
        for j, qq in enumerate(samples):
            i, sc = oracle.flat_i8_query(q[:m], s[:m], qq, k, nthreads=threads)
            best[j] = oracle.merge_hits([best[j], (np.asarray(i, np.int64) + r0, sc)], k)
        ix.upload_rows(r0, q[:m], s[:m])
    ix.upload_finish()
    widx = np.full((len(samples), k), -1, np.int64)
    wsc = np.zeros((len(samples), k), np.float32)
    for j, (i, sc) in enumerate(best):
        widx[j, :len(i)] = i
        wsc[j, :len(sc)] = np.asarray(sc, np.float32)
    return ix, widx, wsc


def _check_batch(ix, Q, k, widx, wsc, rows, what):
    gidx, gsc = ix.topk_arrays(Q, k)
    assert_same(gidx[rows].astype(np.int64), gsc[rows], widx, wsc, what)


def test_c3_full_size_batch_4096(backend):
    """C3: 50M rows of d = 1024 (the mixture recipe bench.py uses), K = 100,
    one batch of 4096 queries on the tensor-core GEMM path."""
    n, d, k, M = 50_000_000, 1024, 100, 4096
    r = synth.Recipe(synth.MIXTURE, d, seed=20263, ncl=10_000, sigma=0.25)
    Q = r.queries(M)
    rows = [0, M - 1]
    ix, widx, wsc = _build_with_oracle(backend, r, n, d, Q[rows], k)
    _check_batch(ix, Q, k, widx, wsc, rows, "C3 full size, batch 4096")
    ix.Close()


def test_c5_full_size_batch_1024(backend):
    """C5: 100M rows of the ties recipe (codes in {-2..2}, scale 1/127), K =
    1000, one batch of 1024 queries: heavy exact ties at the threshold of every
    range, resolved to the lower index over the whole corpus."""
    n, d, k, M = 100_000_000, 256, 1000, 1024
    r = synth.Recipe(synth.TIES, d, seed=20265)
    Q = r.queries(M)
    rows = [0, M - 1]
    ix, widx, wsc = _build_with_oracle(backend, r, n, d, Q[rows], k)
    _check_batch(ix, Q, k, widx, wsc, rows, "C5 full size, batch 1024")
    ix.Close()


def test_c2_full_size_batch_64_and_1(backend):
    """C2: 10M rows of d = 768 (mixture of 1000 clusters, sigma 0.3), K = 100:
    a batch of 64 on the HBM-bound GEMM path, and its first query alone on the
    batch-1 scan, both against the oracle."""
    n, d, k, M = 10_000_000, 768, 100, 64
    r = synth.Recipe(synth.MIXTURE, d, seed=20260, ncl=1000, sigma=0.3)
    Q = r.queries(M)
    rows = [0, M - 1]
    ix, widx, wsc = _build_with_oracle(backend, r, n, d, Q[rows], k)
    _check_batch(ix, Q, k, widx, wsc, rows, "C2 full size, batch 64")
    gidx, gsc = ix.topk_arrays(Q[:1], k)
    assert_same(gidx.astype(np.int64), gsc, widx[:1], wsc[:1], "C2 full size, batch 1")
    ix.Close()


def test_c4_full_shard_batch_512_and_1(backend):
    """C4's per-GPU shard: 25M rows of d = 1024 (unit recipe), K = 10,
    overquery 100 (a 1000-row shortlist). A batch of 512 prefiltered on the
    tensor cores and its first query alone on the popcount pass, both against
    FlatBinaryI8.Query on the CPU. The oracle cuts each block's prefilterHist
    shortlist together with the running one back to the cand nearest under
    (distance, id), which is the global shortlist because the cut decomposes,
    and reranks it at the end (flat_binary_i8.go:86-153)."""
    n, d, k, over, M = 25_000_000, 1024, 10, 100, 512
    cand = k * over
    r = synth.Recipe(synth.UNIT, d, seed=20264)
    ctr = r.center(CHUNK)  # the prefilter's centre: the mean of the first block
    Q = r.queries(M)
    rows = [0, M - 1]
    qc = [oracle.pack_row(q, ctr) for q in Q[rows]]
    keep = [None] * len(rows)  # per sampled query: (ids, codes, int8 rows, scales)
    bix = backend.NewBinaryI8IndexEmpty(n, d, ctr, over)
    for r0 in range(0, n, CHUNK):
        m = min(CHUNK, n - r0)
        bits, bq, bs = r.binary(m, ctr, row0=r0)
        for j in range(len(rows)):
            ids = oracle.prefilter_hist(qc[j], bits, d, cand)
            part = (ids + r0, bits[ids], bq[ids], bs[ids])
            if keep[j] is not None:
                part = tuple(np.concatenate([a, b]) for a, b in zip(keep[j], part))
                sel = oracle.prefilter_hist(qc[j], part[1], d, cand)  # ascending: ids stay in order
                part = tuple(a[sel] for a in part)
            keep[j] = part
        bix.upload_rows(r0, bits, bq, bs)
    bix.upload_finish()
    widx = np.full((len(rows), k), -1, np.int64)
    wsc = np.zeros((len(rows), k), np.float32)
    for j, q in enumerate(Q[rows]):
        gids, bits, bq, bs = keep[j]
        # the shortlist is the whole candidate set: FlatI8's exact top-k over it
        i, sc = oracle.flat_binary_i8_query(bits, ctr, bq, bs, cand, q, k)
        widx[j, :len(i)] = gids[np.asarray(i, np.int64)]
        wsc[j, :len(sc)] = np.asarray(sc, np.float32)
    bix.set_tensor_prefilter(16)
    gidx, gsc = bix.topk_arrays(Q, k)
    assert_same(gidx[rows].astype(np.int64), gsc[rows], widx, wsc, "C4 shard, batch 512")
    gidx, gsc = bix.topk_arrays(Q[:1], k)
    assert_same(gidx.astype(np.int64), gsc, widx[:1], wsc[:1], "C4 shard, batch 1")
    bix.Close()
