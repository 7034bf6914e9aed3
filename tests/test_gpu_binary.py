"""GPU parity for the FlatBinaryI8 device path (sign-bit Hamming prefilter +
int8 rerank) through the C ABI, against the CPU oracle's restatement of
ann/flat_binary_i8.go and ann/flat_binary_prefilter.go.

Re-expresses the reference's FlatBinaryI8 tests: the rerank is bit-identical to
FlatI8 when nothing is pruned (ann/flat_binary_i8_test.go:56), the exact
fallback boundaries k <= 0 / k >= n / cand >= n (:16), all-ties -> [0..k-1]
(ann/flat_binary_test.go:434), and the shortlist equals prefilterHist's
(ids ascending, ties by id) exactly.
"""
import numpy as np
import pytest

import oracle
from aikit_b200 import DeclinedError, synth
from aikit_b200.ann import unpack_keys

pytestmark = pytest.mark.gpu


def build(r, n, centered=True):
    """The reference's newFlatBinaryI8 on the CPU: float rows -> center,
    packed sign codes (prefilter) and int8 rows + scales (FlatI8)."""
    v = r.floats(n)
    ctr = oracle.center(v) if centered else None
    codes = oracle.pack_codes(v, ctr)
    bq, bs = oracle.quantize_rows(v)
    return v, ctr, codes, bq, bs


def oracle_query(codes, ctr, bq, bs, over, q, k):
    i, s = oracle.flat_binary_i8_query(codes, ctr, bq, bs, over, q, k)
    idx = np.full(k, -1, np.int64)
    sc = np.zeros(k, np.float32)
    idx[:len(i)] = i
    sc[:len(s)] = np.asarray(s, np.float32)
    return idx, sc


def check_queries(bix, codes, ctr, bq, bs, over, Q, k, what):
    gidx, gsc = bix.topk_arrays(Q, k)
    for m, q in enumerate(Q):
        widx, wsc = oracle_query(codes, ctr, bq, bs, over, q, k)
        assert gidx[m].astype(np.int64).tolist() == widx.tolist(), f"{what}: query {m} indices"
        ok = widx >= 0
        assert gsc[m][ok].tobytes() == wsc[ok].tobytes(), f"{what}: query {m} scores"


@pytest.mark.parametrize("n,d,over,k,M", [
    (20000, 1024, 16, 10, 3),   # the C4 row shape (128-byte codes: specialised kernel)
    (30000, 768, 16, 10, 2),    # 96-byte codes: generic pitch
    (15000, 384, 8, 25, 2),
    (12000, 2048, 4, 20, 1),    # 256-byte codes
    (5000, 100, 10, 7, 4),      # 2 words: 16-byte pitch, trailing bits cleared
    (4000, 64, 5, 5, 1),        # 1 word, padded to 2
    (40000, 256, 100, 10, 1),   # the C4 over-query (cand 1000)
])
def test_binary_matches_oracle(backend, n, d, over, k, M):
    r = synth.Recipe(synth.MIXTURE, d, seed=n + d, ncl=40, sigma=0.3)
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    Q = r.queries(M)
    check_queries(bix, codes, ctr, bq, bs, over, Q, k, f"n={n} d={d} over={over} k={k}")
    bix.Close()


def test_binary_uncentred(backend):
    r = synth.Recipe(synth.UNIT, 512, seed=9)
    n = 8000
    v, ctr, codes, bq, bs = build(r, n, centered=False)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], None, bq, bs, n, 512, 8)
    check_queries(bix, codes, None, bq, bs, 8, r.queries(3), 12, "uncentred")
    bix.Close()


def test_binary_shortlist_is_prefilter_hist(backend):
    """The device shortlist is prefilterHist's candidate set, exactly."""
    import torch
    r = synth.Recipe(synth.MIXTURE, 1024, seed=77, ncl=20, sigma=0.4)
    n, cand = 50000, 500
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, 1024, 50)
    Q = r.queries(4)
    qd = torch.from_numpy(Q).cuda()
    keys = torch.zeros((4, cand), dtype=torch.int64, device="cuda")
    stream = torch.cuda.Stream()
    bix.prefilter_async(qd.data_ptr(), 4, cand, keys.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    bix.sync()
    gidx, gsc = unpack_keys(keys.cpu().numpy().view(np.uint64))
    for m in range(4):
        qc = oracle.pack_row(Q[m], ctr)
        want = oracle.prefilter_hist(qc, codes, 1024, cand)
        assert sorted(gidx[m].tolist()) == want.tolist()
        # keys carry -distance: sorted by (distance asc, id asc)
        dist = oracle.hamming_rows(qc, codes)
        assert (-gsc[m]).astype(np.int64).tolist() == dist[gidx[m]].astype(np.int64).tolist()
    bix.Close()


def test_binary_nothing_to_prune_is_flat_i8(backend):
    """cand >= n: FlatI8's exact scan (flat_binary_i8.go:95-97), bit-identical."""
    r = synth.Recipe(synth.UNIT, 128, seed=4)
    n = 900
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, 128, 100)  # cand = 10 * 100 >= 900
    Q = r.queries(3)
    gidx, gsc = bix.topk_arrays(Q, 10)
    for m, q in enumerate(Q):
        i, s = oracle.flat_i8_query(bq, bs, q, 10)
        assert gidx[m].tolist() == list(i)
        assert gsc[m].tobytes() == np.asarray(s, np.float32).tobytes()
    bix.Close()


def test_binary_rerank_equals_flat_i8_when_shortlist_covers(backend):
    """A shortlist holding the true top-k reranks to exactly FlatI8's answer
    (ann/flat_binary_i8_test.go:56)."""
    r = synth.Recipe(synth.MIXTURE, 256, seed=12, ncl=5, sigma=0.2)
    n = 3000
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, 256, 200)  # cand 2000 < n
    Q = r.queries(2)
    check_queries(bix, codes, ctr, bq, bs, 200, Q, 10, "wide shortlist")
    bix.Close()


def test_binary_all_ties_identity(backend):
    """Every row identical: every distance and score ties, so the answer is
    [0..k-1] (ann/flat_binary_test.go:434)."""
    d, n, k = 256, 5000, 10
    row = synth.Recipe(synth.UNIT, d, seed=1).floats(1)
    v = np.repeat(row, n, axis=0)
    ctr = oracle.center(v)
    codes = oracle.pack_codes(v, ctr)
    bq, bs = oracle.quantize_rows(v)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, 16)
    gidx, _ = bix.topk_arrays(row, k)
    assert gidx[0].tolist() == list(range(k))
    bix.Close()


def test_binary_declines(backend):
    r = synth.Recipe(synth.UNIT, 64, seed=2)
    n = 1000
    v, ctr, codes, bq, bs = build(r, n)
    bix = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, 64, 0)  # overquery 0 -> 1
    assert bix.overquery == 1
    for k in (0, -1, n, n + 5):
        with pytest.raises(DeclinedError):
            bix.topk_arrays(r.queries(1), k)
    check_queries(bix, codes, ctr, bq, bs, 1, r.queries(2), 5, "overquery 1")
    bix.Close()


def test_binary_row_shards_global_shortlist(backend):
    """Sharded rows: per-shard prefilter, merged shortlist (the global cand
    nearest), per-shard rerank, merged top-k == the unsharded reference."""
    import torch
    d, n, k, over = 512, 30000, 10, 20
    cand = k * over
    r = synth.Recipe(synth.MIXTURE, d, seed=123, ncl=30, sigma=0.35)
    v, ctr, codes, bq, bs = build(r, n)
    bounds = [0, 7001, 19000, n]
    shards = [backend.NewBinaryI8Index(codes[a:b], codes.shape[1], ctr, bq[a:b], bs[a:b], b - a, d, over,
                                       id_base=a) for a, b in zip(bounds[:-1], bounds[1:])]
    M = 3
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
    for m in range(M):
        widx, wsc = oracle_query(codes, ctr, bq, bs, over, Q[m], k)
        assert gidx[m].astype(np.int64).tolist() == widx.tolist()
        assert gsc[m].tobytes() == wsc.tobytes()
    for b in shards:
        b.Close()
