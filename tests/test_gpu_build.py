"""GPU parity for the corpus build on the device (NewFlatI8 and
newFlatBinaryI8 from float rows) against the oracle's restatement of
QuantizeRowInt8 (linalg/quant.go:43-71), the float64 centring
(ann/flat_binary_prefilter.go:64-85) and PackSignBitsRow
(linalg/hamming.go:28-37): every code, scale, centre value and sign word is
bit-identical, and queries on the built index equal the oracle's.
"""
import numpy as np
import pytest

import oracle
from aikit_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,d", [(50000, 384), (3001, 100), (1000, 1024), (257, 17)])
def test_device_quantize_matches_oracle(backend, n, d):
    v = synth.Recipe(synth.MIXTURE, d, seed=n, ncl=7, sigma=0.3).floats(n)
    v[5] = 0.0                      # all-zero row: scale 1
    v[7, 3] = np.nan                # NaN ignored by max|v|, code 0
    v[9] *= 1e-30                   # tiny (subnormal-range) scale
    ix = backend.NewI8IndexFromFloats(v)
    bq, bs = ix.read_rows()
    wq, ws = oracle.quantize_rows(v)
    assert bq.tobytes() == wq.tobytes()
    assert bs.tobytes() == ws.tobytes()
    ix.Close()


@pytest.mark.parametrize("n,d,with_valid", [(60000, 768, False), (20001, 1024, True), (999, 70, True)])
def test_device_binary_build_matches_oracle(backend, n, d, with_valid):
    r = synth.Recipe(synth.MIXTURE, d, seed=n + d, ncl=9, sigma=0.35)
    v = r.floats(n)
    valid = None
    if with_valid:
        valid = (np.random.default_rng(n).random(n) > 0.1).astype(np.uint8)
    bix = backend.NewBinaryI8IndexFromFloats(v, overquery=16, valid=valid)
    ctr = oracle.center(v, valid)
    got = bix.center()
    assert got is not None and got.tobytes() == ctr.tobytes()
    assert bix.read_codes().tobytes() == oracle.pack_codes(v, ctr, valid).tobytes()
    bq, bs = bix.read_rows()
    wq, ws = oracle.quantize_rows(v)
    assert bq.tobytes() == wq.tobytes() and bs.tobytes() == ws.tobytes()
    # the built index answers as the oracle does on the oracle-built corpus
    codes = oracle.pack_codes(v, ctr, valid)
    Q = r.queries(2)
    gi, gs = bix.topk_arrays(Q, 10)
    for m in range(2):
        i, s = oracle.flat_binary_i8_query(codes, ctr, wq, ws, 16, Q[m], 10)
        assert gi[m].tolist() == list(i)
        assert gs[m].tobytes() == np.asarray(s, np.float32).tobytes()
    bix.Close()


def test_device_binary_build_uncentred_and_given_centre(backend):
    r = synth.Recipe(synth.UNIT, 256, seed=3)
    v = r.floats(5000)
    b0 = backend.NewBinaryI8IndexFromFloats(v, centered=False)
    assert b0.center() is None
    assert b0.read_codes().tobytes() == oracle.pack_codes(v, None).tobytes()
    b0.Close()
    # a row shard takes the whole corpus's centre
    full = r.floats(20000)
    ctr = oracle.center(full)
    b1 = backend.NewBinaryI8IndexFromFloats(full[7000:12000], center=ctr, id_base=7000)
    assert b1.center().tobytes() == ctr.tobytes()
    assert b1.read_codes().tobytes() == oracle.pack_codes(full[7000:12000], ctr).tobytes()
    b1.Close()
    # no valid row: no centre (the reference leaves center nil)
    b2 = backend.NewBinaryI8IndexFromFloats(v[:100], valid=np.zeros(100, np.uint8))
    assert b2.center() is None
    assert not b2.read_codes().any()
    b2.Close()
