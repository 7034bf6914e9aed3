"""Pins the CPU oracle (oracle/, the C restatement of the reference's Go path)
against the reference's own literal vectors, known-answer relations and
real-data fixtures. CPU only.

Each test names the reference test it re-expresses.
"""
import json
import os

import numpy as np
import pytest

import oracle
from aikit_b200 import synth

from conftest import GOLDEN


def unit(n, d, seed):
    return synth.Recipe(synth.UNIT, d, seed=seed).floats(n)


# --- linalg/hamming_test.go ---------------------------------------------------

def test_pack_sign_bits_bit_order():
    """TestPackSignBitsRow_bitOrder (linalg/hamming_test.go:12-48): the literal
    golden words, zero packs as 1, the ragged last word's unused bits clear."""
    v = np.full(130, -1, np.float32)
    v[[0, 63, 64, 129]] = 1
    got = oracle.pack_row(v)
    want = np.array([1 | (1 << 63), 1, 1 << 1], np.uint64)
    assert got.tolist() == want.tolist()
    v[2] = 0
    got = oracle.pack_row(v)
    assert int(got[0]) & (1 << 2), "zero must pack as a 1 bit"
    assert int(got[2]) >> 2 == 0, "trailing bits of the ragged last word must be clear"


@pytest.mark.parametrize("words", [1, 2, 3, 4, 5, 8, 12, 13, 16])
@pytest.mark.parametrize("n", [1, 7, 64])
def test_hamming_rows_matches_scalar(words, n):
    """TestHammingRows_matchesScalar (linalg/hamming_test.go:50-80), with an
    independent bit-clearing popcount as the scalar reference."""
    rng = np.random.default_rng(38 + words * 100 + n)
    q = rng.integers(0, 2**64, size=words, dtype=np.uint64)
    codes = rng.integers(0, 2**64, size=(n, words), dtype=np.uint64)
    got = oracle.hamming_rows(q, codes)
    for i in range(n):
        want = 0
        for j in range(words):
            x = int(codes[i, j]) ^ int(q[j])
            while x:
                x &= x - 1
                want += 1
        assert int(got[i]) == want


# --- linalg/quant_test.go -----------------------------------------------------

@pytest.mark.parametrize("d", [1, 3, 15, 16, 17, 63, 64, 65, 100, 384, 768, 1029])
def test_dot_i8_matches_scalar(d):
    """TestDotI8_matchesScalar (linalg/quant_test.go:234): the AVX2 bulk plus
    scalar tail equals the scalar loop, including saturating-magnitude codes."""
    rng = np.random.default_rng(d)
    for a, b in [
        (rng.integers(-127, 128, d, dtype=np.int8), rng.integers(-127, 128, d, dtype=np.int8)),
        (np.full(d, -127, np.int8), np.full(d, -127, np.int8)),
        (np.full(d, 127, np.int8), np.full(d, -127, np.int8)),
    ]:
        want = int(np.dot(a.astype(np.int64), b.astype(np.int64)))
        assert oracle.dot_i8(a, b) == want
        assert oracle.dot_i8(a, b, scalar=True) == want


def test_quantize_zero_row_scales():
    """quantizeRowInt8Core (linalg/quant.go:43-71): all-zero rows get scale 1
    for corpus rows (QuantizeRowInt8) and the sentinel 0 for queries."""
    z = np.zeros(32, np.float32)
    q, s = oracle.quantize_row(z, 1.0)
    assert s == 1.0 and not q.any()
    q, s = oracle.quantize_row(z, 0.0)
    assert s == 0.0 and not q.any()


def test_quantize_round_half_away_and_clamp():
    """math.Round is half away from zero; codes clamp to +-127."""
    row = np.array([127.0, -127.0, 0.5, -0.5, 1.5, -1.5, 2.5, 0.0], np.float32)
    q, s = oracle.quantize_row(row, 1.0)
    assert s == np.float32(1.0)
    assert q.tolist() == [127, -127, 1, -1, 2, -2, 3, 0]


def test_quantize_round_trip():
    """TestQuantizeRowsInt8_roundTrip (linalg/quant_test.go:23): per-element
    reconstruction error within half a quantization step."""
    v = unit(200, 96, 3)
    q, s = oracle.quantize_rows(v)
    rec = q.astype(np.float32) * s[:, None]
    assert np.all(np.abs(rec - v) <= s[:, None] * 0.5 + 1e-7)


def test_w8a8_close_to_f32():
    """TestMatmulBTW8A8_closeToF32 (linalg/quant_test.go:280): relL2 <= 5e-2."""
    rng = np.random.default_rng(5)
    for M, K, N in [(1, 640, 1024), (1, 2048, 640), (4, 256, 300)]:
        a = rng.standard_normal((M, K)).astype(np.float32)
        b = rng.standard_normal((N, K)).astype(np.float32)
        want = a @ b.T
        bq, bs = oracle.quantize_rows(b)
        aq, as_ = oracle.quantize_queries(a)
        got = oracle.w8a8(aq, as_, bq, bs)
        e = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert e <= 5e-2


def test_w8a8_zero_query_scores_zero():
    """w8a8Span's aScales[i]==0 skip (linalg/quant.go:291-294): exactly +0."""
    bq, bs = oracle.quantize_rows(unit(50, 32, 1))
    aq, as_ = oracle.quantize_queries(np.zeros((1, 32), np.float32))
    got = oracle.w8a8(aq, as_, bq, bs)
    assert np.all(got == 0) and not np.signbit(got).any()


def test_w8a8_threads_inert():
    """parallelSpawnCols is numerically inert (linalg/linalg.go:208-233)."""
    bq, bs = oracle.quantize_rows(unit(3001, 77, 2))
    aq, as_ = oracle.quantize_queries(unit(3, 77, 9))
    a = oracle.w8a8(aq, as_, bq, bs, nthreads=1)
    b = oracle.w8a8(aq, as_, bq, bs, nthreads=7)
    assert a.tobytes() == b.tobytes()


# --- topk/topk_test.go, ann/flat_i8.go topHits --------------------------------

def test_top_hits_first_seen_ties():
    """TestSelector_tieBreakFirstSeen (topk/topk_test.go:207-242) through
    topHits: among equal scores the lower index survives."""
    idx, sc = oracle.top_hits(np.array([5, 5, 10], np.float32), 2)
    assert idx.tolist() == [2, 0] and sc.tolist() == [10.0, 5.0]
    idx, _ = oracle.top_hits(np.array([1, 1, 1, 1, 1, 100], np.float32), 3)
    assert idx.tolist() == [5, 0, 1]


def test_top_hits_nan_rejected():
    """TestPush_NaN_Rejected (topk/topk_test.go:111)."""
    s = np.array([np.nan, 1.0, np.nan, 0.5, np.nan], np.float32)
    idx, sc = oracle.top_hits(s, 3)
    assert idx.tolist() == [1, 3]


def test_top_hits_all_ties_identity():
    """All-ties -> ids 0..k-1 (gpu/anncuda/backend_test.go:343)."""
    idx, sc = oracle.top_hits(np.full(1000, 0.25, np.float32), 17)
    assert idx.tolist() == list(range(17))


def test_top_hits_k_semantics():
    """k<=0 or k>=n returns everything, sorted (ann/flat_i8.go:215-224)."""
    s = np.array([0.1, 0.7, 0.7, -2.0], np.float32)
    for k in (0, -1, 4, 99):
        idx, _ = oracle.top_hits(s, k)
        assert idx.tolist() == [1, 2, 0, 3]


def test_top_hits_matches_sort():
    rng = np.random.default_rng(1)
    s = rng.integers(-20, 20, 5000).astype(np.float32)  # heavy ties
    for k in (1, 10, 100, 4999):
        idx, sc = oracle.top_hits(s, k)
        order = sorted(range(len(s)), key=lambda i: (-float(s[i]), i))[:k]
        assert idx.tolist() == order


# --- ann/flat_i8_test.go -------------------------------------------------------

def test_flat_i8_query_semantics():
    """TestFlatI8_topKAndDeterminism (ann/flat_i8_test.go:69-116)."""
    v = unit(200, 64, 4)
    bq, bs = oracle.quantize_rows(v)
    q = unit(1, 64, 5)[0]
    a = oracle.flat_i8_query(bq, bs, q, 10)
    b = oracle.flat_i8_query(bq, bs, q, 10)
    assert a[0].tolist() == b[0].tolist() and a[1].tolist() == b[1].tolist()
    assert np.all(np.diff(a[1]) <= 0)
    assert len(oracle.flat_i8_query(bq, bs, q, -1)[0]) == 200
    assert len(oracle.flat_i8_query(bq, bs, q, 999)[0]) == 200
    assert oracle.flat_i8_query(bq, bs, np.zeros(63, np.float32), 5) is None
    assert oracle.flat_i8_query(np.zeros((0, 0), np.int8), np.zeros(0, np.float32),
                                np.zeros(0, np.float32), 5) is None


def test_flat_i8_recall_vs_float():
    """TestFlatI8_recallVsFlat (ann/flat_i8_test.go:34): int8 top-10 recall vs
    exact float cosine stays high on unit vectors."""
    v = unit(2000, 64, 6)
    bq, bs = oracle.quantize_rows(v)
    Q = unit(20, 64, 7)
    hits = 0
    for q in Q:
        exact = set(np.argsort(-(v @ q), kind="stable")[:10].tolist())
        got = set(oracle.flat_i8_query(bq, bs, q, 10)[0].tolist())
        hits += len(exact & got)
    assert hits / 200 >= 0.9


@pytest.mark.parametrize("mode", ["random", "identical", "twolevel"])
def test_shard_merge_matches_serial(mode):
    """TestFlatQuery_shardedMatchesSerial (ann/flat_shard_test.go:23-61): the
    per-shard top-k + (score desc, id asc) merge equals the serial scan, on
    all-identical and two-level tie corpora and a ragged last shard."""
    n, d = 4097, 96
    if mode == "random":
        v = unit(n, d, 8)
    elif mode == "identical":
        v = np.repeat(unit(1, d, 8), n, axis=0)
    else:
        base = unit(2, d, 8)
        v = base[np.arange(n) % 2]
    bq, bs = oracle.quantize_rows(v)
    q = unit(1, d, 9)[0]
    aq, as_ = oracle.quantize_queries(q[None])
    scores = oracle.w8a8(aq, as_, bq, bs)[0]
    for k in (1, 5, 10, 64):
        want = oracle.top_hits(scores, k)
        for shards in (2, 3, 8):
            bounds = np.linspace(0, n, shards + 1).astype(int)
            parts = []
            for lo, hi in zip(bounds[:-1], bounds[1:]):
                i, s = oracle.top_hits(scores[lo:hi], k)
                parts.append((i + lo, s))
            got = oracle.merge_hits(parts, k)
            assert got[0].tolist() == want[0].tolist() and got[1].tolist() == want[1].tolist()


# --- ann/flat_binary*_test.go ---------------------------------------------------

def _binary_index(v, over):
    c = oracle.center(v)
    codes = oracle.pack_codes(v, c)
    bq, bs = oracle.quantize_rows(v)
    return codes, c, bq, bs


def test_binary_hist_and_heap_agree():
    """TestFlatBinary_histAndHeapAgree (ann/flat_binary_test.go:399): the
    histogram selection equals the heap selection (with an always-live keep)."""
    r = synth.Recipe(synth.MIXTURE, 64, seed=21, ncl=60, sigma=0.5)
    for n, dim in [(3000, 64)]:
        v = r.floats(n)
        c = oracle.center(v)
        codes = oracle.pack_codes(v, c)
        for qi in range(4):
            qc = oracle.pack_row(r.queries(4)[qi], c)
            for cand in (2, 10, 80, 320):
                h = oracle.prefilter_hist(qc, codes, dim, cand)
                for shards in (1, 5):
                    p = oracle.prefilter_heap(qc, codes, dim, cand, np.ones(n, np.uint8), shards)
                    assert h.tolist() == p.tolist()


def test_binary_hist_tie_break_is_by_id():
    """TestFlatBinary_histTieBreakIsByID (ann/flat_binary_test.go:434): an
    all-identical corpus returns ids 0..k-1."""
    v = np.repeat(unit(1, 64, 7), 1000, axis=0)
    codes, c, bq, bs = _binary_index(v, 4)
    got = oracle.flat_binary_i8_query(codes, c, bq, bs, 4, v[0], 10)
    assert got[0].tolist() == list(range(10))


def test_binary_i8_exact_when_nothing_to_prune():
    """TestFlatBinaryI8_exactWhenNothingToPrune (ann/flat_binary_i8_test.go:16)."""
    v = unit(300, 64, 38)
    q = unit(1, 64, 99)[0]
    codes, c, bq, bs = _binary_index(v, 4)
    for over, k in [(4, 0), (4, -1), (4, 300), (400, 5), (60, 5)]:
        want = oracle.flat_i8_query(bq, bs, q, k)
        got = oracle.flat_binary_i8_query(codes, c, bq, bs, over, q, k)
        assert got[0].tolist() == want[0].tolist() and got[1].tolist() == want[1].tolist()


def test_binary_i8_rerank_scores_match_flat_i8():
    """TestFlatBinaryI8_rerankScoresMatchFlatI8 (ann/flat_binary_i8_test.go:56):
    every rerank score is bit-identical to FlatI8's score for that document."""
    v = unit(5000, 128, 380)
    codes, c, bq, bs = _binary_index(v, 16)
    for qi in range(5):
        q = unit(1, 128, 1000 + qi)[0]
        idx, sc = oracle.flat_binary_i8_query(codes, c, bq, bs, 16, q, 10)
        assert len(idx) == 10
        full = dict(zip(*oracle.flat_i8_query(bq, bs, q, 5000)))
        for i, s in zip(idx.tolist(), sc.tolist()):
            assert full[i] == s
        assert np.all(np.diff(sc) <= 0)


def test_center_float64_sequential_and_ragged():
    """newBinaryPrefilter's centre (ann/flat_binary_prefilter.go:64-85) skips
    ragged rows and leaves their codes zero."""
    v = unit(10, 8, 3)
    valid = np.ones(10, np.uint8)
    valid[4] = 0
    c = oracle.center(v, valid)
    want = (v[valid == 1].astype(np.float64).sum(0) / 9).astype(np.float32)
    assert c.tobytes() == want.tobytes()
    codes = oracle.pack_codes(v, c, valid)
    assert not codes[4].any()
    assert oracle.center(v, np.zeros(10, np.uint8)) is None


# --- real-data fixtures ----------------------------------------------------------

def test_retrieval_eval_recall_floor():
    """ann/retrieval_eval_test.go:118-131 on the committed embeddings: FlatI8
    recall@10 against the curated relevance stays within 0.05 of exact float
    Flat's."""
    z = np.load(os.path.join(GOLDEN, "retrieval_eval.npz"))
    docs, qs, rel = z["docs"], z["queries"], z["relevant"]
    bq, bs = oracle.quantize_rows(docs)

    def recall(search):
        tot = 0.0
        for i, q in enumerate(qs):
            r = set(x for x in rel[i].tolist() if x >= 0)
            got = search(q)
            tot += len(r & set(got)) / min(len(r), 10)
        return tot / len(qs)

    flat = recall(lambda q: sorted(range(len(docs)), key=lambda j: (-float(docs[j] @ q), j))[:10])
    i8 = recall(lambda q: oracle.flat_i8_query(bq, bs, q, 10)[0].tolist())
    assert i8 >= flat - 0.05


def test_oracle_reproduces_committed_goldens():
    """The committed seeded goldens (tests/golden/flat_i8_cases.json) still
    come out of the generator + oracle unchanged."""
    import hashlib
    cases = json.load(open(os.path.join(GOLDEN, "flat_i8_cases.json")))
    for name, c in cases.items():
        extra = dict(ncl=c["ncl"], sigma=c["sigma"]) if c["kind"] == synth.MIXTURE else {}
        r = synth.Recipe(c["kind"], c["d"], seed=c["seed"], **extra)
        bq, bs = r.codes(c["n"])
        assert hashlib.sha256(bq.tobytes()).hexdigest() == c["codes_sha256"], name
        Q = r.queries(c["nq"])
        for m in range(c["nq"]):
            i, s = oracle.flat_i8_query(bq, bs, Q[m], c["k"])
            assert i.tolist() == c["idx"][m][:len(i)], name
            assert s.tolist() == c["score"][m][:len(s)], name


def test_oracle_reproduces_reference_kernel_outputs():
    """Reference-run outputs: the reference's own CUDA kernels
    (gpu/anncuda/gemv_w8a8.cu, compiled for sm_100a from its source and run on
    a B200 by tests/golden/make_ref_gpu_golden.py, launched as
    gpu/anncuda/backend.go does) scored and selected these inputs. The
    oracle's W8A8 (linalg/quant.go:248-298) must give the same score matrix
    byte for byte, and its topHits (ann/flat_i8.go:214-246) the same ids and
    float32 scores: the reference's device path is the one its own tests hold
    equal to the Go path (gpu/anncuda/backend_test.go:44, :306)."""
    z = np.load(os.path.join(GOLDEN, "ref_anncuda_outputs.npz"))
    names = sorted({f.split("/")[0] for f in z.files})
    assert len(names) == 4
    for name in names:
        g = lambda key: z[f"{name}/{key}"]
        scores = oracle.w8a8(g("qi8"), g("qscale"), g("codes"), g("scales"))
        assert scores.tobytes() == g("scores").tobytes(), name
        k = int(g("k"))
        for m in range(scores.shape[0]):
            i, sc = oracle.top_hits(scores[m], k)
            assert list(i) == g("idx")[m].astype(np.int64).tolist(), (name, m)
            assert np.asarray(sc, np.float32).tobytes() == g("val")[m].tobytes(), (name, m)


def test_synth_quantizer_matches_oracle():
    v = synth.Recipe(synth.MIXTURE, 200, seed=4, ncl=10, sigma=0.3).floats(500)
    v[3] = 0
    q1, s1 = oracle.quantize_rows(v)
    for i in range(len(v)):
        q2, s2 = synth.quantize_row(v[i])
        assert q2.tobytes() == q1[i].tobytes() and s2 == s1[i]


def test_synth_binary_corpus_matches_oracle():
    """The bench's FlatBinaryI8 generator (no float rows kept) produces the
    oracle's packed sign codes and int8 rows for the same floats; its centre is
    the float64 column mean (block-summed)."""
    r = synth.Recipe(synth.MIXTURE, 200, seed=8, ncl=6, sigma=0.3)
    n = 9000
    v = r.floats(n)
    ctr = r.center(n)
    want_ctr = (v.astype(np.float64).sum(axis=0) / n).astype(np.float32)
    assert np.abs(ctr.astype(np.float64) - want_ctr).max() <= 1e-7
    bits, q, s = r.binary(n, ctr)
    assert bits.tobytes() == oracle.pack_codes(v, ctr).tobytes()
    bq, bs = oracle.quantize_rows(v)
    assert q.tobytes() == bq.tobytes() and s.tobytes() == bs.tobytes()


def test_binary_query_worker_split_is_result_identical():
    """prefilterHist's worker split (flat_binary_prefilter.go:147-178) only
    partitions rows and sums histograms: the threaded oracle returns exactly
    the single-threaded answer."""
    r = synth.Recipe(synth.UNIT, 256, seed=12)
    n = 150_000  # n * words = 600K >= 2^17: the split engages
    ctr = r.center(n)
    bits, q8, sc = r.binary(n, ctr)
    for m, q in enumerate(r.queries(3)):
        a = oracle.flat_binary_i8_query(bits, ctr, q8, sc, 50, q, 10, nthreads=1)
        b = oracle.flat_binary_i8_query(bits, ctr, q8, sc, 50, q, 10, nthreads=7)
        assert a[0].tolist() == b[0].tolist() and a[1].tobytes() == b[1].tobytes(), m
