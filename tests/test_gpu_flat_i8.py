"""GPU parity for the FlatI8 scan (libfi8_b200.so through the C ABI) against
the CPU oracle. Re-expresses gpu/anncuda/backend_test.go's device tests:
exact top-k indices AND bit-identical float32 scores (the W8A8 multiply order
is reproduced, so no tolerance is needed), ties by lower index.
"""
import json
import os
import threading

import numpy as np
import pytest

import oracle
from aikit_b200 import DeclinedError, fi8_format, synth
from aikit_b200.ann import unpack_keys

from conftest import GOLDEN
from parity_util import assert_same, oracle_topk

pytestmark = pytest.mark.gpu


def test_committed_goldens(backend):
    """The seeded goldens (tests/golden/flat_i8_cases.json), incl. K=300 ties."""
    cases = json.load(open(os.path.join(GOLDEN, "flat_i8_cases.json")))
    for name, c in cases.items():
        extra = dict(ncl=c["ncl"], sigma=c["sigma"]) if c["kind"] == synth.MIXTURE else {}
        r = synth.Recipe(c["kind"], c["d"], seed=c["seed"], **extra)
        bq, bs = r.codes(c["n"])
        Q = r.queries(c["nq"])
        ix = backend.NewI8Index(bq, bs, c["n"], c["d"])
        gidx, gsc = ix.topk_arrays(Q, c["k"])
        widx = np.array(c["idx"], np.int64)
        wsc = np.array(c["score"], np.float64).astype(np.float32)
        assert_same(gidx.astype(np.int64), gsc, widx, wsc, name)
        ix.Close()


@pytest.mark.parametrize("n,d", [(1, 1), (31, 3), (257, 16), (1000, 17), (4097, 96), (3000, 100),
                                 (2000, 384), (1500, 768), (700, 1029), (300, 2048)])
def test_score_batch_bit_identical(backend, n, d):
    """ScoreBatch == MatmulBTW8A8 per element, bit for bit (off-block shapes,
    d % 4 != 0 and d < 16 as in TestCUDA_shapesOffBlockBoundary)."""
    r = synth.Recipe(synth.UNIT, d, seed=n + d)
    bq, bs = r.codes(n)
    Q = r.queries(3)
    ix = backend.NewI8Index(bq, bs, n, d)
    dst = np.empty(3 * n, np.float32)
    ix.ScoreBatch(Q, dst)
    aq, as_ = oracle.quantize_queries(Q)
    want = oracle.w8a8(aq, as_, bq, bs)
    assert dst.reshape(3, n).tobytes() == want.tobytes()
    one = np.empty(n, np.float32)
    ix.Score(Q[1], one)
    assert one.tobytes() == want[1].tobytes()
    ix.Close()


def test_topk_c1_config(backend):
    """BASELINE configs[0] (C1): N=100k, d=384 iid N(0,1) unit vectors, K=10,
    batch-1 queries; 256 of its 1000 queries against the oracle."""
    r = synth.Recipe(synth.UNIT, 384, seed=1)
    bq, bs = r.codes(100_000)
    Q = r.queries(256)
    ix = backend.NewI8Index(bq, bs, 100_000, 384)
    gidx = np.empty((256, 10), np.int32)
    gsc = np.empty((256, 10), np.float32)
    for m in range(256):  # batch 1, as the config issues them
        i, s = ix.topk_arrays(Q[m:m + 1], 10)
        gidx[m], gsc[m] = i[0], s[0]
    widx, wsc = oracle_topk(bq, bs, Q, 10)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, "C1")
    ix.Close()


@pytest.mark.parametrize("k", [1, 10, 100, 1000])
def test_topk_k_range(backend, k):
    r = synth.Recipe(synth.MIXTURE, 256, seed=k, ncl=40, sigma=0.3)
    n = 60_000
    bq, bs = r.codes(n)
    Q = r.queries(3)
    ix = backend.NewI8Index(bq, bs, n, 256)
    gidx, gsc = ix.topk_arrays(Q, k)
    widx, wsc = oracle_topk(bq, bs, Q, k)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, f"k={k}")
    ix.Close()


def test_topk_all_ties(backend):
    """TestCUDATopK_tieBreak (gpu/anncuda/backend_test.go:343): every row
    identical -> ids 0..k-1, for k below and above one CTA's tile."""
    v = synth.Recipe(synth.UNIT, 64, seed=2).floats(1)
    bq1, bs1 = oracle.quantize_rows(v)
    n = 70_000
    bq = np.repeat(bq1, n, axis=0)
    bs = np.repeat(bs1, n)
    ix = backend.NewI8Index(bq, bs, n, 64)
    for k in (1, 10, 64, 500, 2000):
        gidx, gsc = ix.topk_arrays(v, k)
        assert gidx[0].tolist() == list(range(k))
        assert np.all(gsc == gsc[0, 0])
    ix.Close()


def test_topk_heavy_ties_c5_recipe(backend):
    """The C5 recipe (codes in {-2..2}, scale 1/127, integer queries) at K=1000."""
    r = synth.Recipe(synth.TIES, 256, seed=5)
    n = 200_000
    bq, bs = r.codes(n)
    Q = r.queries(3)
    ix = backend.NewI8Index(bq, bs, n, 256)
    gidx, gsc = ix.topk_arrays(Q, 1000)
    widx, wsc = oracle_topk(bq, bs, Q, 1000)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, "ties")
    ix.Close()


def test_zero_query(backend):
    """An all-zero query has scale 0 and scores exactly +0 everywhere
    (linalg/quant.go:291-294), so the top-k is ids 0..k-1."""
    bq, bs = synth.Recipe(synth.UNIT, 48, seed=3).codes(5000)
    ix = backend.NewI8Index(bq, bs, 5000, 48)
    gidx, gsc = ix.topk_arrays(np.zeros((1, 48), np.float32), 7)
    assert gidx[0].tolist() == list(range(7))
    assert np.all(gsc == 0) and not np.signbit(gsc).any()
    ix.Close()


def test_nan_and_negative_zero_scores(backend):
    """Hostile scales (a NaN-scaled row, as a corrupt FI8 blob could carry) are
    never returned, like topk's NaN rejection; an underflowing negative score
    keeps its -0.0 bits."""
    n, d = 3000, 32
    bq, bs = synth.Recipe(synth.UNIT, d, seed=4).codes(n)
    bs = bs.copy()
    bs[[5, 77, 1500]] = np.nan
    bs[[9, 10]] = np.float32(1e-38)
    ix = backend.NewI8Index(bq, bs, n, d)
    Q = synth.Recipe(synth.UNIT, d, seed=4).queries(4)
    Q[1] = -bq[9].astype(np.float32)  # strongly negative dot with rows 9, 10
    gidx, gsc = ix.topk_arrays(Q, 2999)
    widx, wsc = oracle_topk(bq, bs, Q, 2999)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, "nan")
    # Score output keeps amd64 NaN bits: a NaN scale propagates its payload, and
    # an Inf query component (scale Inf, all codes 0) makes 0*Inf = 0xFFC00000.
    Q[2, 0] = np.inf
    for m in (1, 2):
        dst = np.empty(n, np.float32)
        ix.Score(Q[m], dst)
        aq, as_ = oracle.quantize_queries(Q[m:m + 1])
        assert dst.tobytes() == oracle.w8a8(aq, as_, bq, bs)[0].tobytes(), m
    ix.Close()


def test_declines(backend):
    """TestCUDATopK declines (gpu/anncuda/backend_test.go:457): k <= 0 and
    k >= n are refused, not approximated."""
    bq, bs = synth.Recipe(synth.UNIT, 16, seed=5).codes(100)
    ix = backend.NewI8Index(bq, bs, 100, 16)
    q = np.zeros((1, 16), np.float32)
    for k in (0, -3, 100, 101):
        with pytest.raises(DeclinedError):
            ix.topk_arrays(q, k)
    assert ix.TopKBatch([q[0]], 99)[0][0].Index == 0
    ix.Close()


def test_wrong_dim_is_an_error(backend):
    from aikit_b200 import Fi8Error
    bq, bs = synth.Recipe(synth.UNIT, 16, seed=5).codes(100)
    ix = backend.NewI8Index(bq, bs, 100, 16)
    with pytest.raises(Fi8Error):
        ix.TopKBatch([np.zeros(15, np.float32)], 5)
    ix.Close()


def test_concurrent_calls(backend):
    """TestCUDA concurrent Score (gpu/anncuda/backend_test.go:246): one index
    shared by several threads returns each caller its own exact answer."""
    r = synth.Recipe(synth.UNIT, 128, seed=6)
    bq, bs = r.codes(20_000)
    Q = r.queries(16)
    ix = backend.NewI8Index(bq, bs, 20_000, 128)
    widx, wsc = oracle_topk(bq, bs, Q, 10)
    errs = []

    def work(t):
        try:
            for rep in range(5):
                m = (t + rep) % 16
                i, s = ix.topk_arrays(Q[m:m + 1], 10)
                assert i[0].tolist() == widx[m].tolist()
                assert s[0].tobytes() == wsc[m].tobytes()
        except Exception as e:  # pragma: no cover - reported below
            errs.append(e)

    ts = [threading.Thread(target=work, args=(t,)) for t in range(8)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs, errs[0]
    ix.Close()


def test_row_shards_merge_equals_whole(backend):
    """Row shards with global ids (id_base) and the device key merge equal the
    whole-corpus answer: the merge rule of queryBatchSharded
    (ann/backend.go:262-277), run here as the multi-GPU merge runs it."""
    import torch
    r = synth.Recipe(synth.MIXTURE, 192, seed=7, ncl=30, sigma=0.3)
    n, k, M = 90_001, 50, 5
    bq, bs = r.codes(n)
    Q = r.queries(M)
    bounds = [0, 20_000, 20_001, 61_234, n]
    shards = [backend.NewI8Index(bq[lo:hi], bs[lo:hi], hi - lo, 192, id_base=lo)
              for lo, hi in zip(bounds[:-1], bounds[1:])]
    dq = torch.from_numpy(Q).cuda()
    keys = torch.zeros((len(shards), M, k), dtype=torch.int64, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    st = stream.cuda_stream
    for s, ix in enumerate(shards):  # shard 1 has a single row (< k): it yields that row
        ix.topk_async(dq.data_ptr(), M, k, keys[s].data_ptr(), st)
    out = torch.zeros((M, k), dtype=torch.int64, device="cuda")
    backend.ctx.merge_keys_async(keys.data_ptr(), len(shards), M, k, out.data_ptr(), st)
    torch.cuda.synchronize()
    for ix in shards:
        ix.sync()
    gidx, gsc = unpack_keys(out.cpu().numpy().view(np.uint64))
    torch.cuda.set_stream(torch.cuda.default_stream())
    widx, wsc = oracle_topk(bq, bs, Q, k)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, "shards")
    for ix in shards:
        ix.Close()


def test_real_embedded_corpus(backend):
    """Real Model2Vec codes (head of the reference's shipped FI8 blob): its own
    dequantized rows and random unit queries, exact against the oracle."""
    q, s = fi8_format.load(open(os.path.join(GOLDEN, "embedded_corpus_head.fi8"), "rb").read())
    n, d = q.shape
    ix = backend.NewI8Index(q, s, n, d)
    Q = np.concatenate([q[[0, 17, 511]].astype(np.float32) * s[[0, 17, 511], None],
                        synth.Recipe(synth.UNIT, d, seed=9).queries(5)])
    gidx, gsc = ix.topk_arrays(Q, 50)
    widx, wsc = oracle_topk(q, s, Q, 50)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, "embedded")
    ix.Close()


def test_retrieval_eval_fixture(backend):
    z = np.load(os.path.join(GOLDEN, "retrieval_eval.npz"))
    docs, qs = z["docs"], z["queries"]
    bq, bs = oracle.quantize_rows(docs)
    ix = backend.NewI8Index(bq, bs, len(docs), docs.shape[1])
    gidx, gsc = ix.topk_arrays(qs, 10)
    widx, wsc = oracle_topk(bq, bs, qs, 10)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, "retrieval_eval")
    ix.Close()


def test_large_c2_shape_sampled(backend):
    """C2's row shape (d=768, mixture of 1000 clusters, sigma 0.3, K=100) at
    N=2M: device top-K of 4 queries against the oracle's full scan."""
    r = synth.Recipe(synth.MIXTURE, 768, seed=2, ncl=1000, sigma=0.3)
    n = 2_000_000
    bq, bs = r.codes(n)
    Q = r.queries(4)
    ix = backend.NewI8Index(bq, bs, n, 768)
    gidx, gsc = ix.topk_arrays(Q, 100)
    widx, wsc = oracle_topk(bq, bs, Q, 100)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, "C2-sample")
    ix.Close()


def test_back_to_back_async_queries(backend):
    """Batch-1 queries launched back to back on one stream with no host sync:
    each scan may start on SMs the previous scan frees while that scan's last
    CTA is still merging, so it must not take the previous query's threshold.
    Queries alternate between full-scale and 1/100-scale vectors, so a stale
    threshold from the previous query would be far above every score of the
    next one."""
    import torch
    from aikit_b200.ann import unpack_keys
    n, d, k, M = 300_000, 256, 50, 24
    r = synth.Recipe(synth.MIXTURE, d, seed=11, ncl=40, sigma=0.3)
    bq, bs = r.codes(n)
    ix = backend.NewI8Index(bq, bs, n, d)
    Q = r.queries(M)
    Q[1::2] *= np.float32(0.01)
    qd = torch.from_numpy(Q).cuda()
    keys = torch.zeros((M, k), dtype=torch.int64, device="cuda")
    st = torch.cuda.Stream()
    torch.cuda.synchronize()
    for m in range(M):
        ix.topk_async(qd[m].data_ptr(), 1, k, keys[m].data_ptr(), st.cuda_stream)
    st.synchronize()
    ix.sync()
    gi, gs = unpack_keys(keys.cpu().numpy().view(np.uint64))
    for m in range(M):
        i, s = oracle.flat_i8_query(bq, bs, Q[m], k)
        assert gi[m].tolist() == list(i), m
        assert gs[m].tobytes() == np.asarray(s, np.float32).tobytes(), m
    ix.Close()
