"""FI8 v1 blob handling (ann/flat_i8_persist.go), CPU only. Re-expresses
ann/flat_i8_persist_test.go and pins the real-data fixtures."""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

import oracle
from aikit_b200 import fi8_format, synth

from conftest import GOLDEN


def _good(n=100, d=32):
    bq, bs = synth.Recipe(synth.UNIT, d, seed=3).codes(n)
    return fi8_format.dumps(bq, bs), bq, bs


def test_round_trip():
    """TestFlatI8_roundTrip (ann/flat_i8_persist_test.go:24)."""
    blob, bq, bs = _good(500, 64)
    q2, s2 = fi8_format.load(blob)
    assert q2.tobytes() == bq.tobytes() and s2.tobytes() == bs.tobytes()
    assert fi8_format.dumps(q2, s2) == blob


def test_empty_round_trip():
    """TestFlatI8_emptyRoundTrip (ann/flat_i8_persist_test.go:53)."""
    blob = fi8_format.dumps(np.zeros((0, 0), np.int8), np.zeros(0, np.float32))
    q, s = fi8_format.load(blob)
    assert q.shape[0] == 0 and s.shape[0] == 0


def test_rejects_bad_blobs():
    """TestLoadFlatI8_rejectsBadBlobs (ann/flat_i8_persist_test.go:71)."""
    good, _, _ = _good()
    flip = bytearray(good)
    flip[0] = (flip[0] + 1) & 0xFF
    for blob in [bytes([1, 2, 3]), b"", bytes(flip), good[:-4], good + b"\0"]:
        with pytest.raises(fi8_format.FormatError):
            fi8_format.load(blob)
    fi8_format.load(good)


def test_rejects_inconsistent_shape():
    """TestLoadFlatI8_rejectsInconsistentShape (ann/flat_i8_persist_test.go:14)
    and the committed fuzz-corpus seed (ann/testdata/fuzz/FuzzLoadFlatI8)."""
    b = struct.pack("<IIIi", fi8_format.MAGIC, fi8_format.VERSION, 0x7FF90000, 0)
    with pytest.raises(fi8_format.FormatError):
        fi8_format.load(b)
    seed = open(os.path.join(GOLDEN, "fuzz_seed_flati8.bin"), "rb").read()
    assert len(seed) == 16
    with pytest.raises(fi8_format.FormatError):
        fi8_format.load(seed)


def test_negative_shape_rejected():
    b = struct.pack("<IIii", fi8_format.MAGIC, fi8_format.VERSION, -4, 2) + bytes(100)
    with pytest.raises(fi8_format.FormatError):
        fi8_format.load(b)


def test_mmap_matches_copy(tmp_path):
    """TestLoadFlatI8Mmap equals LoadFlatI8 (ann/flat_i8_mmap_test.go:26)."""
    blob, bq, bs = _good(300, 48)
    p = tmp_path / "x.fi8"
    p.write_bytes(blob)
    q, s = fi8_format.load_mmap(str(p))
    assert np.array_equal(q, bq) and np.array_equal(s, bs)


def test_embedded_corpus_fixture():
    """The reference's shipped real-data blob: header (d=256, n=1747) recorded
    at fixture generation; the committed 512-row head re-parses and serves a
    FlatI8 query whose rank-0 hit is the row itself or, when the corpus holds an
    exact duplicate (rows 432 and 511 here), the lower-index duplicate."""
    meta = json.load(open(os.path.join(GOLDEN, "embedded_corpus_meta.json")))
    assert (meta["dim"], meta["n"]) == (256, 1747)
    assert meta["bytes"] == 16 + meta["n"] * meta["dim"] + 4 * meta["n"]
    blob = open(os.path.join(GOLDEN, "embedded_corpus_head.fi8"), "rb").read()
    q, s = fi8_format.load(blob)
    assert q.shape == (512, 256)
    # a dequantized row as the query: it must rank itself first
    for row in (0, 17, 511):
        qv = q[row].astype(np.float32) * s[row]
        idx, sc = oracle.flat_i8_query(q, s, qv, 5)
        assert idx[0] <= row and q[idx[0]].tobytes() == q[row].tobytes()
        if idx[0] != row:
            assert row in idx.tolist() and sc[idx.tolist().index(row)] == sc[0]


def test_paged_block_rows_follow_the_reference():
    """pagedBlockRows (ann/flat_i8_mmap.go:46-56): about 1 MiB of codes per
    block, at least one row."""
    assert fi8_format.paged_block_rows(1024) == 1024
    assert fi8_format.paged_block_rows(768) == (1 << 20) // 768
    assert fi8_format.paged_block_rows(1 << 21) == 1
    assert fi8_format.paged_block_rows(0) == 1


class _FakeIndex:
    def __init__(self, n, dim):
        self.n, self.dim, self.rows, self.finished = n, dim, [], False
        self.codes = np.zeros((n, dim), np.int8)
        self.scales = np.zeros(n, np.float32)

    def upload_rows(self, row0, codes, scales):
        c = np.asarray(codes, np.int8).reshape(-1, self.dim)
        self.codes[row0:row0 + len(c)] = c
        self.scales[row0:row0 + len(c)] = scales
        self.rows.append((row0, len(c)))

    def upload_finish(self):
        self.finished = True


class _FakeBackend:
    def NewI8IndexEmpty(self, n, dim, id_base=0):
        self.ix = _FakeIndex(n, dim)
        return self.ix


@pytest.mark.parametrize("n,dim,block", [(1000, 300, 77), (4096, 256, 0), (5, 1, 2)])
def test_upload_paged_walks_blocks_in_order(tmp_path, n, dim, block):
    """upload_paged (the paged-index device path): every row once, in blocks
    of block_rows (pagedBlockRows when 0) in ascending order, a ragged last
    block, then the finish call; the uploaded rows equal the blob's."""
    rng = np.random.default_rng(n)
    bq = rng.integers(-127, 128, size=(n, dim), dtype=np.int8)
    bs = rng.random(n).astype(np.float32)
    path = tmp_path / "c.fi8"
    path.write_bytes(fi8_format.dumps(bq, bs))
    be = _FakeBackend()
    ix = fi8_format.upload_paged(be, str(path), block_rows=block)
    rows = block or fi8_format.paged_block_rows(dim)
    want = [(r0, min(rows, n - r0)) for r0 in range(0, n, rows)]
    assert ix.rows == want and ix.finished
    assert ix.codes.tobytes() == bq.tobytes() and ix.scales.tobytes() == bs.tobytes()


def test_upload_paged_rejects_bad_blobs(tmp_path):
    empty = tmp_path / "empty.fi8"
    empty.write_bytes(b"")
    with pytest.raises(fi8_format.FormatError):
        fi8_format.upload_paged(_FakeBackend(), str(empty))
    zero = tmp_path / "zero.fi8"
    zero.write_bytes(fi8_format.dumps(np.zeros((0, 0), np.int8), np.zeros(0, np.float32)))
    with pytest.raises(fi8_format.FormatError):
        fi8_format.upload_paged(_FakeBackend(), str(zero))
    bad = tmp_path / "bad.fi8"
    bad.write_bytes(b"\x00" * 20)
    with pytest.raises(fi8_format.FormatError):
        fi8_format.upload_paged(_FakeBackend(), str(bad))
