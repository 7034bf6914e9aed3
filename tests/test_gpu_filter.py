"""GPU parity for the keep filter (QueryFilter) through the C ABI, against the
oracle's keep-aware restatements: FlatI8.QueryFilter = topHits with keep
(ann/flat_i8.go:136, :214-246) and FlatBinaryI8.QueryFilter = prefilterHeap +
rerank (ann/flat_binary_i8.go:83, flat_binary_prefilter.go:227-313). The
device takes the filter as a bitmap over global row ids.
"""
import numpy as np
import pytest

import oracle
from aikit_b200 import synth
from aikit_b200.ann import keep_bitmap, unpack_keys

from parity_util import assert_same

pytestmark = pytest.mark.gpu


def oracle_filtered(bq, bs, Q, k, keep):
    idx = np.full((len(Q), k), -1, np.int64)
    sc = np.zeros((len(Q), k), np.float32)
    for m, q in enumerate(Q):
        i, s = oracle.flat_i8_query(bq, bs, q, k, keep=keep.astype(np.uint8))
        idx[m, :len(i)] = i
        sc[m, :len(s)] = np.asarray(s, np.float32)
    return idx, sc


@pytest.mark.parametrize("n,d,M,k,frac", [
    (60000, 384, 1, 10, 0.3),      # batch 1: the fused scan
    (60000, 384, 12, 10, 0.3),     # batched: the GEMM epilogue
    (40000, 768, 64, 100, 0.05),   # C2 shape, a sparse filter
    (5000, 100, 3, 50, 0.005),     # fewer kept rows than k: -1 padding
])
def test_flat_i8_query_filter(backend, n, d, M, k, frac):
    r = synth.Recipe(synth.MIXTURE, d, seed=n + M, ncl=20, sigma=0.3)
    bq, bs = r.codes(n)
    Q = r.queries(M)
    keep = np.random.default_rng(n).random(n) < frac
    ix = backend.NewI8Index(bq, bs, n, d)
    gi, gs = ix.topk_arrays(Q, k, keep=keep)
    wi, ws = oracle_filtered(bq, bs, Q, k, keep)
    assert_same(gi.astype(np.int64), gs, wi, ws, f"filtered n={n} M={M} k={k}")
    # the unfiltered call on the same index is unaffected
    gi2, _ = ix.topk_arrays(Q[:1], k)
    wi2, _ = oracle_filtered(bq, bs, Q[:1], k, np.ones(n, bool))
    assert gi2[0].tolist() == wi2[0].tolist()
    ix.Close()


def test_filter_drops_the_best_rows_and_short_bitmaps(backend):
    """Filtering out the unfiltered top-k returns the next rows; a bitmap
    shorter than n keeps nothing past its end; an all-false filter returns
    nothing."""
    r = synth.Recipe(synth.UNIT, 256, seed=6)
    n, k = 30000, 20
    bq, bs = r.codes(n)
    Q = r.queries(5)
    ix = backend.NewI8Index(bq, bs, n, 256)
    top, _ = ix.topk_arrays(Q, k)
    keep = np.ones(n, bool)
    keep[top.reshape(-1)] = False
    gi, gs = ix.topk_arrays(Q, k, keep=keep)
    assert_same(gi.astype(np.int64), gs, *oracle_filtered(bq, bs, Q, k, keep), "drop best")
    short = np.ones(n // 2, bool)
    gi, gs = ix.topk_arrays(Q, k, keep=short)
    full = np.zeros(n, bool)
    full[: n // 2] = True
    assert_same(gi.astype(np.int64), gs, *oracle_filtered(bq, bs, Q, k, full), "short bitmap")
    gi, _ = ix.topk_arrays(Q, k, keep=np.zeros(n, bool))
    assert (gi == -1).all()
    ix.Close()


def test_filter_row_shards_global_ids(backend):
    """The bitmap is over global ids: shards (id_base) filter their own rows,
    and the merged answer equals the unsharded filtered one."""
    import torch
    d, n, k, M = 128, 50000, 30, 4
    r = synth.Recipe(synth.MIXTURE, d, seed=99, ncl=10, sigma=0.3)
    bq, bs = r.codes(n)
    Q = r.queries(M)
    keep = np.random.default_rng(5).random(n) < 0.4
    d_keep = torch.from_numpy(keep_bitmap(keep).view(np.int64).copy()).cuda()
    bounds = [0, 17001, 35000, n]
    shards = [backend.NewI8Index(bq[a:b], bs[a:b], b - a, d, id_base=a) for a, b in zip(bounds[:-1], bounds[1:])]
    qd = torch.from_numpy(Q).cuda()
    stream = torch.cuda.Stream()
    parts = torch.zeros((3, M, k), dtype=torch.int64, device="cuda")
    for s, ix in enumerate(shards):
        ix.topk_async(qd.data_ptr(), M, k, parts[s].data_ptr(), stream.cuda_stream, d_keep=d_keep.data_ptr(),
                      keep_nbits=n)
    out = torch.zeros((M, k), dtype=torch.int64, device="cuda")
    backend.ctx.merge_keys_async(parts.data_ptr(), 3, M, k, out.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    for ix in shards:
        ix.sync()
    gi, gs = unpack_keys(out.cpu().numpy().view(np.uint64))
    assert_same(gi.astype(np.int64), gs, *oracle_filtered(bq, bs, Q, k, keep), "sharded filter")
    for ix in shards:
        ix.Close()


@pytest.mark.parametrize("n,d,over,k,frac", [
    (30000, 1024, 16, 10, 0.25),
    (20000, 512, 40, 10, 0.02),   # the filter leaves fewer rows than cand
    (900, 128, 100, 10, 0.5),     # cand >= n: FlatI8's exact filtered scan
])
def test_binary_query_filter(backend, n, d, over, k, frac):
    r = synth.Recipe(synth.MIXTURE, d, seed=n + over, ncl=15, sigma=0.3)
    v = r.floats(n)
    ctr = oracle.center(v)
    codes = oracle.pack_codes(v, ctr)
    bq, bs = oracle.quantize_rows(v)
    keep = np.random.default_rng(over).random(n) < frac
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    Q = r.queries(3)
    gi, gs = bix.topk_arrays(Q, k, keep=keep)
    for m in range(len(Q)):
        i, s = oracle.flat_binary_i8_query(codes, ctr, bq, bs, over, Q[m], k, keep=keep.astype(np.uint8))
        want_i = np.full(k, -1, np.int64)
        want_s = np.zeros(k, np.float32)
        want_i[:len(i)] = i
        want_s[:len(s)] = np.asarray(s, np.float32)
        assert gi[m].astype(np.int64).tolist() == want_i.tolist(), m
        ok = want_i >= 0
        assert gs[m][ok].tobytes() == want_s[ok].tobytes(), m
    bix.Close()
