"""The reference's own device path on the same B200: the kernels of
gpu/anncuda/gemv_w8a8.cu, compiled for sm_100a from the reference source
(oracle/ref_anncuda.py), launched as gpu/anncuda/backend.go launches them.

These pin the oracle and this library to reference-run outputs: the W8A8
scores the reference's GEMV kernels write (ScoreBatch,
gpu/anncuda/backend.go:212-236) equal the oracle's and fi8_score_batch's byte
for byte, and the top-k its selection kernels return (TopKBatch, :568-667:
topk_rows' k passes for k > 64, the register split/merge kernels below) equals
the oracle's FlatI8 answer and fi8_topk_batch's, ids and float32 score bits,
ties by lower index included. The reference's own gate for this is
TestCUDATopK_matchesCPU (gpu/anncuda/backend_test.go:306).
"""
import numpy as np
import pytest

import oracle
from aikit_b200 import synth
from oracle import ref_anncuda

from parity_util import assert_same, oracle_topk

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_anncuda.available(),
                                 reason="oracle/_ref not built (needs the reference source tree at build time)")]


def run_reference(backend, bq, bs, Q, k):
    """Reference kernels: (scores [M][n] f32, idx [M][k] int32, val [M][k] f32)."""
    import torch
    n, d = bq.shape
    M = len(Q)
    aq, as_ = oracle.quantize_queries(Q)  # the reference quantizes on the host (backend.go:270-298)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    codes, scales, qi8, qs = dev(bq), dev(bs), dev(aq), dev(as_)
    scores = torch.empty((M, n), dtype=torch.float32, device="cuda")
    idx = torch.empty((M, k), dtype=torch.int32, device="cuda")
    val = torch.empty((M, k), dtype=torch.float32, device="cuda")
    ref = ref_anncuda.RefTopK(n, d, M, k, backend.ctx.sm_count())
    ref.score(codes.data_ptr(), scales.data_ptr(), qi8.data_ptr(), qs.data_ptr(), scores.data_ptr())
    torch.cuda.synchronize()
    sc = scores.cpu().numpy().copy()
    ref.topk(scores.data_ptr(), idx.data_ptr(), val.data_ptr())
    torch.cuda.synchronize()
    ref.close()
    return sc, idx.cpu().numpy(), val.cpu().numpy()


@pytest.mark.parametrize("n,d,M", [
    (20000, 768, 1),     # gemv_w8a8 (one query), the C2 row shape
    (30001, 100, 3),     # batch8, dim % 4 != 0: the reference's byte path
    (50000, 256, 8),     # batch8, a full 8-query tile
    (40000, 384, 21),    # batch16, two query planes, the second partial
])
def test_reference_scores_equal_oracle_and_ours(backend, n, d, M):
    r = synth.Recipe(synth.MIXTURE, d, seed=n + d, ncl=40, sigma=0.3)
    bq, bs = r.codes(n)
    Q = r.queries(M)
    ref_scores, _, _ = run_reference(backend, bq, bs, Q, 10)
    aq, as_ = oracle.quantize_queries(Q)
    assert ref_scores.tobytes() == oracle.w8a8(aq, as_, bq, bs).tobytes()
    ix = backend.NewI8Index(bq, bs, n, d)
    ours = np.empty(M * n, np.float32)
    ix.ScoreBatch(Q, ours)
    assert ours.tobytes() == ref_scores.tobytes()
    ix.Close()


@pytest.mark.parametrize("n,d,M,k,recipe", [
    (60000, 256, 1, 10, "mixture"),     # topk_split_r16 + topk_merge_r16 (one query over many blocks)
    (60000, 256, 8, 50, "mixture"),     # topk_split_r64 + merge
    (60000, 768, 4, 100, "mixture"),    # k > 64: topk_rows, k block-wide argmax passes
    (80000, 384, 64, 100, "mixture"),   # batch16 planes + topk_rows, the C2 batch shape
    (50000, 256, 6, 100, "ties"),       # the C5 recipe: heavy score ties, lower index first
    (50000, 128, 200, 16, "unit"),      # M above the SM count: topk_rows_r16, one block per query
])
def test_reference_topk_equals_oracle_and_ours(backend, n, d, M, k, recipe):
    if recipe == "ties":
        r = synth.Recipe(synth.TIES, d, seed=n + M)
    elif recipe == "unit":
        r = synth.Recipe(synth.UNIT, d, seed=n + M)
    else:
        r = synth.Recipe(synth.MIXTURE, d, seed=n + M, ncl=50, sigma=0.3)
    bq, bs = r.codes(n)
    Q = r.queries(M)
    _, ridx, rval = run_reference(backend, bq, bs, Q, k)
    widx, wsc = oracle_topk(bq, bs, Q, k)
    assert_same(ridx.astype(np.int64), rval, widx, wsc, f"reference kernels n={n} d={d} M={M} k={k}")
    ix = backend.NewI8Index(bq, bs, n, d)
    gidx, gsc = ix.topk_arrays(Q, k)
    assert gidx.astype(np.int64).tolist() == ridx.astype(np.int64).tolist()
    assert gsc.tobytes() == rval.tobytes()
    ix.Close()
