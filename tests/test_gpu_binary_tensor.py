"""GPU parity for FlatBinaryI8's tensor-core prefilter
(fi8_bin_set_tensor_prefilter) through the C ABI.

The codes are unpacked on the device to +1/-1 int8 rows, so the dot of a
query's sign row with a corpus row is dim - 2 * (Hamming distance) and a
batch's distances are one tcgen05 kind::i8 GEMM. The shortlist it selects must
be prefilterHist's (ann/flat_binary_prefilter.go:145-216) exactly: the same
keys (-distance, global id), bit for bit, as the popcount pass produces, and
the same final answers as the oracle's FlatBinaryI8.Query
(ann/flat_binary_i8.go:86-109), including QueryFilter's keep set
(prefilter.go:227-313), ragged rows, row shards and distance ties at the cut.
"""
import numpy as np
import pytest

import oracle
from aikit_b200 import synth
from aikit_b200.ann import keep_bitmap, unpack_keys

pytestmark = pytest.mark.gpu


def build(r, n, centered=True, valid=None):
    v = r.floats(n)
    ctr = oracle.center(v, valid) if centered else None
    codes = oracle.pack_codes(v, ctr, valid)
    bq, bs = oracle.quantize_rows(v)
    return v, ctr, codes, bq, bs


def shortlist(bix, Q, cand, keep=None):
    """Sorted shortlist keys [M][cand] (uint64) from the device prefilter."""
    import torch
    M = len(Q)
    qd = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    keys = torch.zeros((M, cand), dtype=torch.int64, device="cuda")
    d_keep = None
    if keep is not None:
        d_keep = torch.from_numpy(keep_bitmap(keep).view(np.int64).copy()).cuda()
    stream = torch.cuda.Stream()
    bix.prefilter_async(qd.data_ptr(), M, cand, keys.data_ptr(), stream.cuda_stream, sorted_keys=True,
                        d_keep=d_keep.data_ptr() if d_keep is not None else 0,
                        keep_nbits=len(keep) if keep is not None else 0)
    stream.synchronize()
    bix.sync()
    return keys.cpu().numpy().view(np.uint64)


def oracle_answers(codes, ctr, bq, bs, over, Q, k, keep=None):
    idx = np.full((len(Q), k), -1, np.int64)
    sc = np.zeros((len(Q), k), np.float32)
    kp = keep.astype(np.uint8) if keep is not None else None
    for m, q in enumerate(Q):
        i, s = oracle.flat_binary_i8_query(codes, ctr, bq, bs, over, q, k, keep=kp)
        idx[m, :len(i)] = i
        sc[m, :len(s)] = np.asarray(s, np.float32)
    return idx, sc


def assert_answers(gidx, gsc, widx, wsc, what):
    for m in range(len(widx)):
        assert gidx[m].astype(np.int64).tolist() == widx[m].tolist(), f"{what}: query {m} indices"
        ok = widx[m] >= 0
        assert gsc[m][ok].tobytes() == wsc[m][ok].tobytes(), f"{what}: query {m} scores"


@pytest.mark.parametrize("n,d,M,k,over,centered", [
    (60000, 1024, 64, 10, 100, True),   # the C4 row shape, cand 1000, one 64-query tile
    (30000, 1024, 130, 10, 50, True),   # two 128-query tiles, the second with 2 queries
    (20000, 100, 17, 7, 20, True),      # dim 100: 112-byte sign rows, the K tail zero
    (25000, 512, 9, 12, 30, False),     # uncentred prefilter
    (70000, 64, 40, 10, 100, True),     # 64 bits: most of the cut's distance ties
])
def test_tensor_shortlist_equals_popcount(backend, n, d, M, k, over, centered):
    r = synth.Recipe(synth.MIXTURE, d, seed=n + d + M, ncl=30, sigma=0.35)
    v, ctr, codes, bq, bs = build(r, n, centered)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    Q = r.queries(M)
    cand = k * over
    want = shortlist(bix, Q, cand)          # the popcount pass
    bix.set_tensor_prefilter(1)
    got = shortlist(bix, Q, cand)           # the GEMM
    assert got.tobytes() == want.tobytes(), "tensor shortlist differs from the popcount shortlist"
    gi, gs = unpack_keys(got)
    for m in range(min(M, 3)):
        qc = oracle.pack_row(Q[m], ctr)
        assert sorted(gi[m].tolist()) == oracle.prefilter_hist(qc, codes, d, cand).tolist()
        dist = oracle.hamming_rows(qc, codes)
        assert (-gs[m]).astype(np.int64).tolist() == dist[gi[m]].astype(np.int64).tolist()
    # the whole query through the host entry point
    sub = Q[:4]
    gidx, gsc = bix.topk_arrays(Q, k)
    assert_answers(gidx[:4], gsc[:4], *oracle_answers(codes, ctr, bq, bs, over, sub, k), f"n={n} d={d} M={M}")
    bix.Close()


def test_tensor_prefilter_min_batch_and_release(backend):
    """Batches below min_batch keep the popcount pass; 0 frees the rows; the
    answers never change."""
    d, n, k, over = 256, 20000, 10, 30
    r = synth.Recipe(synth.MIXTURE, d, seed=5, ncl=20, sigma=0.3)
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    Q = r.queries(8)
    base = bix.topk_arrays(Q, k)
    bix.set_tensor_prefilter(4)
    one = bix.topk_arrays(Q[:1], k)            # below min_batch: popcount
    n_pop = bix.last_launch_count()
    many = bix.topk_arrays(Q, k)               # the GEMM
    n_gemm = bix.last_launch_count()
    assert n_pop != n_gemm
    assert one[0].tolist() == base[0][:1].tolist()
    assert many[0].tolist() == base[0].tolist() and many[1].tobytes() == base[1].tobytes()
    bix.set_tensor_prefilter(0)
    again = bix.topk_arrays(Q, k)
    assert again[0].tolist() == base[0].tolist()
    bix.set_tensor_prefilter(2)               # rebuilt after a release
    assert bix.topk_arrays(Q, k)[0].tolist() == base[0].tolist()
    bix.Close()


@pytest.mark.parametrize("frac", [0.3, 0.002])
def test_tensor_prefilter_keep(backend, frac):
    """QueryFilter: the shortlist is the cand nearest kept rows; with fewer
    kept rows than cand, every kept row and empty keys after them."""
    d, n, k, over = 1024, 40000, 10, 50
    r = synth.Recipe(synth.MIXTURE, d, seed=31, ncl=25, sigma=0.35)
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    keep = np.random.default_rng(7).random(n) < frac
    Q = r.queries(20)
    cand = k * over
    want = shortlist(bix, Q, cand, keep=keep)
    bix.set_tensor_prefilter(1)
    got = shortlist(bix, Q, cand, keep=keep)
    assert got.tobytes() == want.tobytes()
    gidx, gsc = bix.topk_arrays(Q, k, keep=keep)
    assert_answers(gidx[:3], gsc[:3], *oracle_answers(codes, ctr, bq, bs, over, Q[:3], k, keep=keep), "keep")
    bix.Close()


def test_tensor_prefilter_ragged_rows_device_build(backend):
    """An index built on the device with ragged (invalid) rows: their codes
    are all zero, i.e. all -1 sign rows, and they stay candidates as in the
    reference."""
    d, n, k, over = 768, 30001, 10, 40
    r = synth.Recipe(synth.MIXTURE, d, seed=17, ncl=20, sigma=0.3)
    valid = (np.random.default_rng(3).random(n) > 0.2).astype(np.uint8)
    v, ctr, codes, bq, bs = build(r, n, valid=valid)
    bix = backend.NewBinaryI8IndexFromFloats(v, overquery=over, valid=valid)
    Q = r.queries(33)
    cand = k * over
    want = shortlist(bix, Q, cand)
    bix.set_tensor_prefilter(1)
    assert shortlist(bix, Q, cand).tobytes() == want.tobytes()
    gidx, gsc = bix.topk_arrays(Q, k)
    assert_answers(gidx[:3], gsc[:3], *oracle_answers(codes, ctr, bq, bs, over, Q[:3], k), "ragged")
    bix.Close()


def test_tensor_prefilter_row_shards(backend):
    """Row shards (id_base): per-shard GEMM shortlists merge into the global
    shortlist; the reranked answer equals the unsharded reference."""
    import torch
    d, n, k, over = 512, 45000, 10, 20
    cand = k * over
    r = synth.Recipe(synth.MIXTURE, d, seed=321, ncl=30, sigma=0.35)
    v, ctr, codes, bq, bs = build(r, n)
    bounds = [0, 11111, 30000, n]
    shards = [backend.NewBinaryI8Index(codes[a:b], codes.shape[1], ctr, bq[a:b], bs[a:b], b - a, d, over,
                                       id_base=a) for a, b in zip(bounds[:-1], bounds[1:])]
    for s in shards:
        s.set_tensor_prefilter(1)
    M = 24
    Q = r.queries(M)
    qd = torch.from_numpy(Q).cuda()
    S = len(shards)
    stream = torch.cuda.Stream()
    short = torch.zeros((S, M, cand), dtype=torch.int64, device="cuda")
    for s, b in enumerate(shards):
        b.prefilter_async(qd.data_ptr(), M, cand, short[s].data_ptr(), stream.cuda_stream)
    gshort = torch.zeros((M, cand), dtype=torch.int64, device="cuda")
    backend.ctx.merge_keys_async(short.data_ptr(), S, M, cand, gshort.data_ptr(), stream.cuda_stream)
    part = torch.zeros((S, M, k), dtype=torch.int64, device="cuda")
    for s, b in enumerate(shards):
        b.rerank_async(qd.data_ptr(), M, gshort.data_ptr(), cand, k, part[s].data_ptr(), stream.cuda_stream)
    out = torch.zeros((M, k), dtype=torch.int64, device="cuda")
    backend.ctx.merge_keys_async(part.data_ptr(), S, M, k, out.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    for b in shards:
        b.sync()
    gidx, gsc = unpack_keys(out.cpu().numpy().view(np.uint64))
    assert_answers(gidx[:4], gsc[:4], *oracle_answers(codes, ctr, bq, bs, over, Q[:4], k), "shards")
    for b in shards:
        b.Close()


@pytest.mark.parametrize("M", [64, 17])
def test_tensor_prefilter_after_stale_tmem(backend, M):
    """A batch of at most 64 queries runs 64-query MMA tiles, which write TMEM
    lanes 0-15 of each 32-lane sub-partition only; the epilogue reads the other
    lanes too. Whatever stale accumulators those lanes hold, they hold no query
    and must yield no candidate. The tensor-pipe probe first leaves large
    accumulators in every SM's TMEM."""
    d, n, k, over = 1024, 30000, 10, 40
    r = synth.Recipe(synth.MIXTURE, d, seed=M + 1, ncl=20, sigma=0.35)
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    Q = r.queries(M)
    cand = k * over
    want = shortlist(bix, Q, cand)
    bix.set_tensor_prefilter(1)
    for _ in range(2):
        backend.ctx.probe_tensor_i8(500)
        assert shortlist(bix, Q, cand).tobytes() == want.tobytes()
    bix.Close()


def test_prefilter_at_the_cand_limit(backend):
    """cand = 2048, the largest shortlist the device takes (k = 16, overquery
    128), on 64-bit codes where hundreds of rows tie at the cut: the GEMM's
    shortlist equals the popcount pass's and the answers equal the oracle's.
    One more k makes cand 2176, which both prefilters decline."""
    from aikit_b200 import DeclinedError
    d, n, k, over = 64, 40000, 16, 128
    r = synth.Recipe(synth.MIXTURE, d, seed=31, ncl=30, sigma=0.35)
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    Q = r.queries(24)
    cand = k * over
    want = shortlist(bix, Q, cand)
    base = bix.topk_arrays(Q, k)
    with pytest.raises(DeclinedError):
        bix.topk_arrays(Q, k + 1)
    bix.set_tensor_prefilter(1)
    assert shortlist(bix, Q, cand).tobytes() == want.tobytes()
    got = bix.topk_arrays(Q, k)
    assert got[0].tolist() == base[0].tolist() and got[1].tobytes() == base[1].tobytes()
    assert_answers(got[0][:3], got[1][:3], *oracle_answers(codes, ctr, bq, bs, over, Q[:3], k), "cand 2048")
    with pytest.raises(DeclinedError):
        bix.topk_arrays(Q, k + 1)
    bix.Close()


@pytest.mark.parametrize("ctas", [1, 7, 146])
def test_tensor_prefilter_grid_sizes(backend, ctas):
    """The Hamming-mode GEMM on a capped persistent grid: 200 queries make two
    128-query tiles (the second with 72), so with an odd G each CTA's query
    tile alternates from unit to unit. The shortlist stays the popcount
    pass's."""
    from aikit_b200._ffi import FI8_OPT_GEMM_CTAS, check, lib
    d, n, k, over = 512, 30000, 10, 20
    r = synth.Recipe(synth.MIXTURE, d, seed=40 + ctas, ncl=20, sigma=0.35)
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    Q = r.queries(200)
    cand = k * over
    want = shortlist(bix, Q, cand)
    bix.set_tensor_prefilter(1)
    check(lib().fi8_index_set_option(bix._ih, FI8_OPT_GEMM_CTAS, ctas))
    assert shortlist(bix, Q, cand).tobytes() == want.tobytes()
    bix.Close()


def test_tensor_prefilter_overflow_is_redone_exactly(backend):
    """A corpus ordered against the first query (every later row nearer to
    it) makes the last row range admit about 324K candidates for that query,
    beyond its 64K-key buffer, so the tensor-core shortlist comes back
    incomplete. The query call notices and redoes the batch with the popcount
    pass: the answers are exact, as the reference's CPU FlatBinaryI8 (which
    has no such buffer) gives them."""
    d, n, k, over = 64, 400_000, 10, 10
    r = synth.Recipe(synth.UNIT, d, seed=12)
    v, ctr, codes, bq, bs = build(r, n)
    Q = r.queries(2)
    dist = oracle.hamming_rows(oracle.pack_row(Q[0], ctr), codes).astype(np.int64)
    order = np.argsort(-dist, kind="stable")  # the nearest rows last
    codes, bq, bs = (np.ascontiguousarray(a[order]) for a in (codes, bq, bs))
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    want = bix.topk_arrays(Q, k)  # the popcount pass
    bix.set_tensor_prefilter(1)
    got = bix.topk_arrays(Q, k)   # the GEMM overflows; the call redoes it
    assert got[0].tolist() == want[0].tolist() and got[1].tobytes() == want[1].tobytes()
    assert_answers(got[0], got[1], *oracle_answers(codes, ctr, bq, bs, over, Q, k), "overflow")
    bix.Close()


def test_tensor_prefilter_async_overflow_is_exact(backend):
    """The device-resident prefilter on the adversarially ordered corpus: the
    popcount redo is gated on the batch's overflow flag and runs in stream
    order, so fi8_bin_prefilter_async's keys are the popcount shortlist's,
    sorted for the cross-shard merge, the sync reports no error, and
    ShardedBinary (one rank here) returns the oracle's answers."""
    import torch
    from aikit_b200.dist import ShardedBinary
    d, n, k, over = 64, 400_000, 10, 10
    r = synth.Recipe(synth.UNIT, d, seed=12)
    v, ctr, codes, bq, bs = build(r, n)
    Q = r.queries(2)
    dist = oracle.hamming_rows(oracle.pack_row(Q[0], ctr), codes).astype(np.int64)
    order = np.argsort(-dist, kind="stable")  # the nearest rows last
    codes, bq, bs = (np.ascontiguousarray(a[order]) for a in (codes, bq, bs))
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    cand = k * over
    want = shortlist(bix, Q, cand)  # the popcount pass
    bix.set_tensor_prefilter(1)
    got = shortlist(bix, Q, cand)   # the GEMM overflows; the gated redo recomputes it
    bix.sync()
    assert got.tobytes() == want.tobytes()
    stream = torch.cuda.Stream()
    qd = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    keys = ShardedBinary(bix, backend.ctx, 1, stream).topk_async(qd.data_ptr(), 2, k)
    stream.synchronize()
    bix.sync()
    gi, gs = unpack_keys(keys.cpu().numpy().view(np.uint64))
    assert_answers(gi, gs, *oracle_answers(codes, ctr, bq, bs, over, Q, k), "async overflow")
    bix.Close()


def test_tensor_prefilter_cta_pair_equals_single(backend):
    """The Hamming-mode GEMM on CTA pairs (batches above 128 queries) gives the
    single-CTA shortlist keys byte for byte."""
    d, n, k, over = 1024, 40000, 10, 100
    r = synth.Recipe(synth.MIXTURE, d, seed=77, ncl=30, sigma=0.35)
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    bix.set_tensor_prefilter(1)
    bix.set_gemm_pair(True)
    Q = r.queries(300)
    pair = shortlist(bix, Q, k * over)
    bix.set_gemm_pair(False)
    single = shortlist(bix, Q, k * over)
    assert pair.tobytes() == single.tobytes()
    got = bix.topk_arrays(Q[:3], k)
    assert_answers(got[0], got[1], *oracle_answers(codes, ctr, bq, bs, over, Q[:3], k), "pair")
    bix.Close()
