"""fi8_topk1_noalloc: the allocation-free single-query top-K.

Some callers cannot allocate device memory while serving: their HBM is
reserved at start-up (the corpus plus a caching allocator's pool), so a
cudaMalloc on the query path could fail, and it may synchronize the whole
device. fi8_topk1_noalloc serves them from a fixed array inside the library.
These tests call it through the C ABI and check that it returns exactly what
the allocating entry point (fi8_topk_batch_async, M = 1) returns, on calls in
a row (the shared array keeps the previous call's contents), and that k above
its limit is a clear error. This file sorts last so a stop-at-first-failure
run has already run every other test.
"""
import numpy as np
import pytest

from aikit_b200 import Fi8Error, synth
from aikit_b200.ann import unpack_keys

from parity_util import assert_same, oracle_topk

pytestmark = pytest.mark.gpu


def _device_keys(ix, q_dev, k, noalloc, stream):
    import torch
    keys = torch.full((k,), -1, dtype=torch.int64, device="cuda")
    if noalloc:
        ix.topk1_noalloc(q_dev.data_ptr(), k, keys.data_ptr(), stream.cuda_stream)
    else:
        ix.topk_async(q_dev.data_ptr(), 1, k, keys.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    ix.sync()
    return keys.cpu().numpy().view(np.uint64).copy()


@pytest.mark.parametrize("k", [10, 256])
def test_noalloc_matches_allocating_entry_point(backend, k):
    import torch
    r = synth.Recipe(synth.MIXTURE, 384, seed=31, ncl=100, sigma=0.3)
    n = 300_000
    bq, bs = r.codes(n)
    Q = r.queries(3)
    ix = backend.NewI8Index(bq, bs, n, 384)
    stream = torch.cuda.Stream()
    qd = [torch.from_numpy(Q[m].copy()).cuda() for m in range(3)]
    want = [_device_keys(ix, qd[m], k, False, stream) for m in range(3)]
    # two calls in a row, then the first query again: the shared scratch must
    # carry nothing from one call into the next
    got = [_device_keys(ix, qd[m], k, True, stream) for m in (0, 1, 0)]
    for g, m in zip(got, (0, 1, 0)):
        assert g.tobytes() == want[m].tobytes()
    gi, gs = unpack_keys(got[0][None, :])
    wi, ws = oracle_topk(bq, bs, Q[:1], k)
    assert_same(gi.astype(np.int64), gs, wi, ws, "noalloc vs oracle")
    ix.Close()


def test_noalloc_rejects_k_beyond_limit(backend):
    import torch
    bq, bs = synth.Recipe(synth.UNIT, 64, seed=2).codes(5000)
    ix = backend.NewI8Index(bq, bs, 5000, 64)
    q = torch.zeros(64, dtype=torch.float32, device="cuda")
    keys = torch.zeros(257, dtype=torch.int64, device="cuda")
    with pytest.raises(Fi8Error, match="allocation-free limit"):
        ix.topk1_noalloc(q.data_ptr(), 257, keys.data_ptr())
    ix.Close()


def test_noalloc_small_index_and_two_indexes_on_one_device(backend):
    """A corpus of a few thousand rows (a scan grid of a handful of CTAs, far
    below the SM count) and a second index on the same device, called one
    after the other on one stream: both share the one array, and each answer
    equals the allocating entry point's and the oracle's."""
    import torch
    stream = torch.cuda.Stream()
    ra = synth.Recipe(synth.UNIT, 128, seed=41)
    rb = synth.Recipe(synth.MIXTURE, 256, seed=42, ncl=20, sigma=0.3)
    aq, as_ = ra.codes(3000)   # ~12 tiles: a few CTAs
    bq, bs = rb.codes(90_000)
    ia = backend.NewI8Index(aq, as_, 3000, 128)
    ib = backend.NewI8Index(bq, bs, 90_000, 256)
    Qa, Qb = ra.queries(2), rb.queries(2)
    for m in range(2):
        for ix, Q, codes, scales, k in ((ia, Qa, aq, as_, 64), (ib, Qb, bq, bs, 100)):
            qd = torch.from_numpy(Q[m].copy()).cuda()
            want = _device_keys(ix, qd, k, False, stream)
            got = _device_keys(ix, qd, k, True, stream)
            assert got.tobytes() == want.tobytes()
            gi, gs = unpack_keys(got[None, :])
            wi, ws = oracle_topk(codes, scales, Q[m:m + 1], k)
            assert_same(gi.astype(np.int64), gs, wi, ws, "noalloc, two indexes")
    ia.Close()
    ib.Close()
