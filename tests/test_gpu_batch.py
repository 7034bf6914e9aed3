"""GPU parity for the batched FlatI8 path (tcgen05 kind::i8 GEMM + exact
threshold selection) through the C ABI, against the CPU oracle. Re-expresses
TestCUDAGEMM_batchMatchesQuery / TestCUDATopK_matchesCPU
(gpu/anncuda/backend_test.go:114, :306, :512): the batch answer equals the
per-query answer exactly (indices and float32 score bits).
"""
import numpy as np
import pytest

import oracle
from aikit_b200 import DeclinedError, synth

from parity_util import assert_same, oracle_topk

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,d,M,k", [
    (3000, 96, 5, 10),        # d % 128 != 0: the last K tile is zero-filled by TMA
    (20000, 768, 64, 100),    # the C2 row shape at batch 64
    (60000, 256, 130, 100),   # two query tiles, the second mostly padding
    (100000, 384, 16, 10),    # the C1 shape, batched
    (50000, 1024, 256, 100),  # the C3 row shape at batch 256
    (2000, 16, 3, 7),
    (700, 1040, 4, 5),        # pitch 1040: 9 K tiles, the last one partial
])
def test_batch_matches_oracle(backend, n, d, M, k):
    r = synth.Recipe(synth.MIXTURE, d, seed=n + M, ncl=50, sigma=0.3)
    bq, bs = r.codes(n)
    Q = r.queries(M)
    ix = backend.NewI8Index(bq, bs, n, d)
    gidx, gsc = ix.topk_arrays(Q, k)
    widx, wsc = oracle_topk(bq, bs, Q, k)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, f"batch n={n} d={d} M={M} k={k}")
    ix.Close()


def test_gemm_equals_scan(backend):
    """Both device paths return identical keys for the same batch (the
    reference's kernelsAgree gate, gpu/anncuda/backend_test.go:583-716)."""
    r = synth.Recipe(synth.UNIT, 256, seed=3)
    n = 120_000
    bq, bs = r.codes(n)
    Q = r.queries(9)
    ix = backend.NewI8Index(bq, bs, n, 256)
    ix.set_gemm_min_batch(1)
    a = ix.topk_arrays(Q, 50)
    one = ix.topk_arrays(Q[:1], 50)
    ix.set_gemm_min_batch(1 << 20)
    b = ix.topk_arrays(Q, 50)
    assert a[0].tolist() == b[0].tolist() and a[1].tobytes() == b[1].tobytes()
    assert one[0][0].tolist() == b[0][0].tolist()
    ix.Close()


def test_batch_ties_k1000(backend):
    """The C5 recipe (codes in {-2..2}, fixed scale, integer queries) at K=1000:
    massive score ties resolved by lower index, exactly."""
    r = synth.Recipe(synth.TIES, 256, seed=5)
    n = 150_000
    bq, bs = r.codes(n)
    Q = r.queries(6)
    ix = backend.NewI8Index(bq, bs, n, 256)
    gidx, gsc = ix.topk_arrays(Q, 1000)
    widx, wsc = oracle_topk(bq, bs, Q, 1000)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, "ties")
    ix.Close()


def test_batch_all_identical_rows(backend):
    v = synth.Recipe(synth.UNIT, 128, seed=2).floats(1)
    bq1, bs1 = oracle.quantize_rows(v)
    n = 40_000
    ix = backend.NewI8Index(np.repeat(bq1, n, axis=0), np.repeat(bs1, n), n, 128)
    Q = np.concatenate([v, -v, np.zeros_like(v)])
    gidx, gsc = ix.topk_arrays(Q, 300)
    for m in range(3):
        assert gidx[m].tolist() == list(range(300))
    ix.Close()


@pytest.mark.parametrize("M", [8, 160])
def test_batch_at_the_top_k_limit(backend, M):
    """k = 4096, the largest k the batched select takes, on tied scores: the
    kept list goes through the shared-memory sort, not the rank placement.
    M = 8 stages each query's union in shared memory; M = 160, more queries
    than SMs, streams the unions from L2. One more k is declined, not
    approximated; a single query takes the scan's own limit."""
    r = synth.Recipe(synth.TIES, 128, seed=M)
    n = 60_000
    bq, bs = r.codes(n)
    Q = r.queries(M)
    ix = backend.NewI8Index(bq, bs, n, 128)
    gidx, gsc = ix.topk_arrays(Q, 4096)
    widx, wsc = oracle_topk(bq, bs, Q, 4096)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, f"k=4096 M={M}")
    with pytest.raises(DeclinedError):
        ix.topk_arrays(Q, 4097)
    k1 = ix.max_k()
    gidx, gsc = ix.topk_arrays(Q[:1], k1)
    widx, wsc = oracle_topk(bq, bs, Q[:1], k1)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, f"batch 1 k={k1}")
    ix.Close()


@pytest.mark.parametrize("ctas", [0, 1, 5, 7, 146])
def test_gemm_grid_sizes(backend, ctas):
    """The answer does not depend on the GEMM's persistent grid (the multi-GPU
    path runs it on all SMs but two). With G CTAs, CTA c takes units c, c+G,
    ..., and a unit's query tile changes from one unit to the next unless G
    is a multiple of the tile count: here 3 tiles of a 300-query batch, the
    last one holding 44 queries. Rows of 256 bytes take the launch's grid
    rule: a cap of 146 (and the default, one CTA per SM) runs on the largest
    multiple of 3 below it, so every CTA keeps one tile; caps of 5 and 7 are
    too far from a multiple and keep the changing tiles."""
    r = synth.Recipe(synth.MIXTURE, 256, seed=ctas, ncl=30, sigma=0.3)
    n = 30_000
    bq, bs = r.codes(n)
    Q = r.queries(300)
    ix = backend.NewI8Index(bq, bs, n, 256)
    ix.set_gemm_ctas(ctas)
    gidx, gsc = ix.topk_arrays(Q, 50)
    widx, wsc = oracle_topk(bq, bs, Q, 50)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, f"ctas={ctas}")
    ix.Close()


def test_batch_overflow_falls_back_exactly(backend):
    """A corpus ordered against the query (every later row beats every earlier
    one) makes a row range admit more candidates than its buffer holds; the
    host API must detect that and still return the exact answer."""
    r = synth.Recipe(synth.UNIT, 64, seed=8)
    n = 400_000
    bq, bs = r.codes(n)
    q = r.queries(2)
    aq, as_ = oracle.quantize_queries(q[:1])
    order = np.argsort(oracle.w8a8(aq, as_, bq, bs)[0], kind="stable")  # ascending score
    bq, bs = np.ascontiguousarray(bq[order]), np.ascontiguousarray(bs[order])
    ix = backend.NewI8Index(bq, bs, n, 64)
    gidx, gsc = ix.topk_arrays(q, 20)
    widx, wsc = oracle_topk(bq, bs, q, 20)
    assert_same(gidx.astype(np.int64), gsc, widx, wsc, "overflow")
    ix.Close()


def _against_query_order(r, n, d):
    """A corpus sorted by ascending score against the first query: every later
    row beats every earlier one, so a row range admits more candidates than
    its buffer holds."""
    bq, bs = r.codes(n)
    q = r.queries(2)
    aq, as_ = oracle.quantize_queries(q[:1])
    order = np.argsort(oracle.w8a8(aq, as_, bq, bs)[0], kind="stable")
    return np.ascontiguousarray(bq[order]), np.ascontiguousarray(bs[order]), q


@pytest.mark.parametrize("M", [2, 70, 300])
def test_async_overflow_is_exact(backend, M):
    """The device-resident form on the same corpus: the gated redo runs in
    stream order, so the keys are exact without a host round trip, the next
    sync reports no error, and ShardedTopK (the multi-GPU path, here one
    rank) hands the exact keys on. Batches of 2 (a 64-query tile), 70 (a
    128-query tile) and 300 (three tiles, and more queries than SMs: the
    redo's one scan launch runs in several waves of one CTA per query)."""
    import torch
    from aikit_b200.ann import unpack_keys
    from aikit_b200.dist import ShardedTopK
    r = synth.Recipe(synth.UNIT, 64, seed=8)
    n, k = 400_000, 20
    bq, bs, q2 = _against_query_order(r, n, 64)
    Q = np.concatenate([q2, r.queries(M, row0=50)])[:M]
    ix = backend.NewI8Index(bq, bs, n, 64)
    stream = torch.cuda.Stream()
    qd = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    keys = torch.zeros((M, k), dtype=torch.int64, device="cuda")
    ix.topk_async(qd.data_ptr(), M, k, keys.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    ix.sync()  # no overflow flag is left for the sync
    sh = ShardedTopK(ix, backend.ctx, 1, stream)
    merged = sh.topk_async(qd.data_ptr(), M, k)
    stream.synchronize()
    ix.sync()
    widx, wsc = oracle_topk(bq, bs, Q, k)
    for got in (keys, merged):
        gi, gs = unpack_keys(got.cpu().numpy().view(np.uint64))
        assert_same(gi.astype(np.int64), gs, widx, wsc, f"async overflow M={M}")
    # the redo ran exactly once per call: its scan launches were opened
    ix.set_kernel_timing(True)
    ix.topk_async(qd.data_ptr(), M, k, keys.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    ix.set_kernel_timing(False)
    kt = ix.kernel_times()
    # queries per gated scan launch: as many as ~32 MB of scratch allows
    kp = 1 << (k - 1).bit_length()
    chunk = min(65535, max(backend.ctx.sm_count(), (32 << 20) // (2 * kp * 8)))
    assert kt["redo_gated"]["launches"] == 1 + (M + chunk - 1) // chunk
    ix.Close()


def test_async_without_overflow_leaves_gate_closed(backend):
    """On an ordinary corpus the gated redo returns at once: the async keys
    equal the oracle's, and each gated launch is short."""
    import torch
    from aikit_b200.ann import unpack_keys
    r = synth.Recipe(synth.MIXTURE, 256, seed=31, ncl=40, sigma=0.3)
    n, M, k = 200_000, 64, 100
    bq, bs = r.codes(n)
    Q = r.queries(M)
    ix = backend.NewI8Index(bq, bs, n, 256)
    stream = torch.cuda.Stream()
    qd = torch.from_numpy(Q).cuda()
    keys = torch.zeros((M, k), dtype=torch.int64, device="cuda")
    ix.set_kernel_timing(True)
    for _ in range(3):
        ix.topk_async(qd.data_ptr(), M, k, keys.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    ix.set_kernel_timing(False)
    kt = ix.kernel_times()
    ix.sync()
    assert kt["redo_gated"]["launches"] == 3 * 2
    # each closed-gate launch only waits for the previous kernel and returns
    # (timed here with an event pair around it, which costs more than the
    # launch itself when the launches chain back to back)
    assert kt["redo_gated"]["ms"] / kt["redo_gated"]["launches"] < 0.1
    gi, gs = unpack_keys(keys.cpu().numpy().view(np.uint64))
    widx, wsc = oracle_topk(bq, bs, Q[:8], k)
    assert_same(gi[:8].astype(np.int64), gs[:8], widx, wsc, "gate closed")
    ix.Close()


def test_batch_row_shard_ids(backend):
    """id_base offsets the returned indices of a shard in the batched path."""
    r = synth.Recipe(synth.UNIT, 192, seed=4)
    bq, bs = r.codes(30_000)
    Q = r.queries(4)
    ix = backend.NewI8Index(bq[10_000:], bs[10_000:], 20_000, 192, id_base=10_000)
    gidx, gsc = ix.topk_arrays(Q, 25)
    widx, wsc = oracle_topk(bq[10_000:], bs[10_000:], Q, 25)
    assert_same(gidx.astype(np.int64), gsc, widx + 10_000, wsc, "shard")
    ix.Close()


@pytest.mark.parametrize("share", [0.5, 0.97])
def test_cpu_gpu_shard_split(backend, share):
    """EnableGPUShardSplit / queryBatchSharded (ann/backend.go:207-346): the
    device index holds the first int(share * n) rows (built from a prefix of
    the corpus, as the reference's NewI8Index call does), the CPU scores the
    rest, and the two shard-local top-k lists merge by (score desc, index asc)
    into exactly the whole corpus's answer."""
    n, d, k = 40_000, 256, 50
    r = synth.Recipe(synth.MIXTURE, d, seed=21, ncl=20, sigma=0.3)
    bq, bs = r.codes(n)
    rows = min(max(int(share * n), 1), n - 1)
    ix = backend.NewI8Index(bq[:rows], bs[:rows], rows, d)
    Q = r.queries(12)
    gidx, gsc = ix.topk_arrays(Q, k)  # the device shard, one batch
    for m, q in enumerate(Q):
        ci, cs = oracle.flat_i8_query(bq[rows:], bs[rows:], q, k)  # the CPU shard
        dev = [(int(i), float(s)) for i, s in zip(gidx[m], gsc[m]) if i >= 0]
        mi, ms = oracle.merge_hits([([i for i, _ in dev], [s for _, s in dev]),
                                    (np.asarray(ci, np.int64) + rows, np.asarray(cs))], k)
        wi, ws = oracle.flat_i8_query(bq, bs, q, k)
        assert mi.tolist() == list(wi)
        assert np.asarray(ms, np.float32).tobytes() == np.asarray(ws, np.float32).tobytes()
    ix.Close()


@pytest.mark.parametrize("n,d,M,k,ctas", [
    (60000, 256, 129, 50, 0),     # one pair unit column: the odd CTA's tile holds one query
    (50000, 1024, 300, 100, 0),   # two pairs, the second partial
    (30000, 96, 1000, 20, 0),     # a zero-filled K tail, four pairs
    (80000, 384, 520, 100, 6),    # three clusters walking many units
    (40000, 512, 260, 64, 2),     # a single cluster
])
def test_cta_pair_equals_single_cta(backend, n, d, M, k, ctas):
    """Batches above 128 queries run on CTA pairs (tcgen05 cta_group::2,
    256-query x 256-row units, FI8_OPT_GEMM_PAIR): keys identical, byte for
    byte, to the single-CTA GEMM and to the oracle on sampled queries."""
    r = synth.Recipe(synth.MIXTURE, d, seed=n + M + d, ncl=60, sigma=0.3)
    bq, bs = r.codes(n)
    Q = r.queries(M)
    ix = backend.NewI8Index(bq, bs, n, d)
    if ctas:
        ix.set_gemm_ctas(ctas)
    ix.set_gemm_pair(True)
    pair = ix.topk_arrays(Q, k)
    ix.set_gemm_pair(False)
    single = ix.topk_arrays(Q, k)
    assert pair[0].tolist() == single[0].tolist() and pair[1].tobytes() == single[1].tobytes()
    rows = [0, M // 2, M - 1]
    widx, wsc = oracle_topk(bq, bs, Q[rows], k)
    assert_same(pair[0][rows].astype(np.int64), pair[1][rows], widx, wsc, f"pair n={n} d={d} M={M}")
    ix.Close()
