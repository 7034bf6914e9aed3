"""GPU tests of the paged / streamed device path: an empty index filled block
by block (fi8_index_create_empty + fi8_index_upload_rows), which is how a paged
FlatI8 (LoadFlatI8MmapPaged, ann/flat_i8_mmap.go:75-102) reaches the device
without ever being resident on the host as a whole. The reference refuses
EnableGPU on a paged index (ann/backend.go:162); its own paged scan is
byte-identical to the resident one (flat_i8_mmap.go:69), and so is this
upload: the rows, the scores and the top-k equal fi8_index_create's.
"""
import numpy as np
import pytest

import oracle
from aikit_b200 import Fi8Error, fi8_format, synth

pytestmark = pytest.mark.gpu


def test_upload_paged_blob_equals_resident(backend, tmp_path):
    d, n, k = 300, 50001, 20
    r = synth.Recipe(synth.MIXTURE, d, seed=808, ncl=25, sigma=0.3)
    bq, bs = r.codes(n)
    path = tmp_path / "corpus.fi8"
    path.write_bytes(fi8_format.dumps(bq, bs))
    ix = fi8_format.upload_paged(backend, str(path), block_rows=777)  # many blocks, a ragged last one
    got_q, got_s = ix.read_rows()
    assert got_q.tobytes() == bq.tobytes() and got_s.tobytes() == bs.tobytes()
    ref = backend.NewI8Index(bq, bs, n, d)
    Q = r.queries(9)
    for m in (9, 1):  # the GEMM path and the batch-1 scan
        gi, gs = ix.topk_arrays(Q[:m], k)
        wi, ws = ref.topk_arrays(Q[:m], k)
        assert gi.tolist() == wi.tolist() and gs.tobytes() == ws.tobytes()
    i, s = oracle.flat_i8_query(bq, bs, Q[0], k)
    assert gi[0].tolist() == list(i)
    ix.Close()
    ref.Close()


def test_upload_rows_any_order_and_unuploaded_rows(backend):
    d, n = 128, 20000
    r = synth.Recipe(synth.UNIT, d, seed=3)
    bq, bs = r.codes(n)
    ix = backend.NewI8IndexEmpty(n, d)
    blocks = [(a, min(a + 3000, n)) for a in range(0, n, 3000)]
    for a, b in reversed(blocks[1:]):  # every block but the first, last one first
        ix.upload_rows(a, bq[a:b], bs[a:b])
    ix.upload_finish()
    q = r.queries(1)[0]
    dst = np.empty(n, np.float32)
    ix.Score(q, dst)
    aq, asc = oracle.quantize_queries(q[None, :])
    full = oracle.w8a8(aq, asc, bq, bs)[0]  # the resident corpus's scores
    assert (dst[:3000] == 0.0).all()  # never uploaded: all-zero rows with scale 0
    assert dst[3000:].tobytes() == full[3000:].tobytes()
    ix.upload_rows(0, bq[:3000], bs[:3000])
    ix.upload_finish()
    ix.Score(q, dst)
    assert dst.tobytes() == full.tobytes()
    with pytest.raises(Fi8Error):
        ix.upload_rows(n - 10, bq[:20], bs[:20])  # past the end
    ix.Close()


def test_binary_streamed_upload_equals_resident(backend):
    """A FlatBinaryI8 shard filled block by block (fi8_bin_index_create_empty +
    fi8_bin_upload_rows, out of order, a ragged last block) holds the same
    codes and rows as fi8_bin_index_create's and answers identically: the
    popcount prefilter, the tensor-core prefilter after the upload, and the
    oracle's FlatBinaryI8.Query (ann/flat_binary_i8.go:86-109)."""
    d, n, k, over = 320, 30001, 10, 20
    r = synth.Recipe(synth.MIXTURE, d, seed=909, ncl=30, sigma=0.35)
    v = r.floats(n)
    ctr = oracle.center(v)
    codes = oracle.pack_codes(v, ctr)
    bq, bs = oracle.quantize_rows(v)
    ix = backend.NewBinaryI8IndexEmpty(n, d, ctr, over)
    blocks = [(a, min(a + 4096, n)) for a in range(0, n, 4096)]
    for a, b in reversed(blocks):
        ix.upload_rows(a, codes[a:b], bq[a:b], bs[a:b])
    ix.upload_finish()
    assert ix.read_codes().tobytes() == codes.tobytes()
    got_q, got_s = ix.read_rows()
    assert got_q.tobytes() == bq.tobytes() and got_s.tobytes() == bs.tobytes()
    ref = backend.NewBinaryI8Index(codes, codes.shape[1], ctr, bq, bs, n, d, over)
    Q = r.queries(20)
    want = ref.topk_arrays(Q, k)
    got = ix.topk_arrays(Q, k)
    assert got[0].tolist() == want[0].tolist() and got[1].tobytes() == want[1].tobytes()
    ix.set_tensor_prefilter(4)
    got = ix.topk_arrays(Q, k)
    assert got[0].tolist() == want[0].tolist() and got[1].tobytes() == want[1].tobytes()
    i, s = oracle.flat_binary_i8_query(codes, ctr, bq, bs, over, Q[0], k)
    assert got[0][0].tolist() == list(i)
    with pytest.raises(Fi8Error):
        ix.upload_rows(0, codes[:10], bq[:10], bs[:10])  # after the sign rows were built
    ix.Close()
    ref.Close()
