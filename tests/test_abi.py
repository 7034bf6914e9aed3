"""The C ABI library loads and exports every symbol include/fi8.h declares.
CPU only: no compute call is made without a GPU."""
import ctypes
import os
import re

from aikit_b200 import _ffi
from aikit_b200.build import build_fi8

from conftest import ROOT


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "fi8.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fi8_[a-z0-9_]+)\s*\(", src)))


def test_library_builds_and_loads():
    path = build_fi8()
    assert os.path.exists(path)
    ctypes.CDLL(path)


def test_exports_every_declared_symbol():
    lib = ctypes.CDLL(build_fi8())
    syms = declared_symbols()
    assert len(syms) >= 10
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_header():
    assert sorted(_ffi.SIGNATURES) == declared_symbols()


def test_keys_unpack_round_trip_host():
    """fi8_keys_unpack is host-only; the key layout orders (score desc, index
    asc) and restores -0.0 exactly."""
    import numpy as np
    from aikit_b200.ann import unpack_keys

    def make_key(score, idx):
        b = np.float32(score).view(np.uint32).item()
        negzero = 1 if b == 0x80000000 else 0
        if b == 0x80000000:
            b = 0
        ordv = (~b & 0xFFFFFFFF) if (b & 0x80000000) else (b | 0x80000000)
        return (ordv << 32) | (((0x7FFFFFFF - idx) & 0x7FFFFFFF) << 1) | negzero

    cases = [(1.5, 0), (1.5, 7), (-0.0, 3), (0.0, 2), (-2.25, 9), (float("inf"), 11), (-1e-38, 5)]
    keys = np.array([make_key(s, i) for s, i in cases] + [0], np.uint64)
    idx, sc = unpack_keys(keys)
    for (s, i), gi, gs in zip(cases, idx[:-1], sc[:-1]):
        assert gi == i and np.float32(s).tobytes() == np.float32(gs).tobytes()
    assert idx[-1] == -1
    order = sorted(range(len(cases)), key=lambda j: -int(keys[j]))
    want = sorted(range(len(cases)), key=lambda j: (-cases[j][0], cases[j][1]))
    assert order == want


def test_purego_adapter_binds_declared_symbols():
    """The cgo-free Go adapter in INTEGRATION.md (purego.RegisterLibFunc, the
    way the reference's gocudrv binds libcuda, gpu/cuda.go:11,54) binds only
    symbols that include/fi8.h declares and the library exports, and covers
    every call the seam's interfaces need: ann.Backend.NewI8Index,
    I8Index.Score/Close, I8BatchIndex.ScoreBatch, I8TopKIndex.TopKBatch
    (ann/backend.go:16-55), QueryFilter, the paged upload and the
    FlatBinaryI8 index."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    start = doc.index("## Go adapter (cgo-free, purego)")
    block = doc[start:doc.index("```\n", doc.index("```go", start) + 5)]
    bound = set(re.findall(r'"(fi8_[a-z0-9_]+)":\s*&fi8\.', block))
    declared = set(declared_symbols())
    assert bound <= declared, sorted(bound - declared)
    lib = ctypes.CDLL(build_fi8())
    assert all(hasattr(lib, s) for s in bound)
    needed = {"fi8_last_error", "fi8_device_count", "fi8_ctx_create", "fi8_index_create", "fi8_index_destroy",
              "fi8_score", "fi8_score_batch", "fi8_topk_batch", "fi8_topk_batch_keep",
              "fi8_index_create_empty", "fi8_index_upload_rows", "fi8_index_upload_finish",
              "fi8_bin_index_create", "fi8_bin_query_topk", "fi8_bin_query_topk_keep",
              "fi8_bin_set_tensor_prefilter", "fi8_bin_index_destroy"}
    assert needed <= bound, sorted(needed - bound)
    # every bound entry point is called through the table somewhere in the doc
    fields = re.findall(r'"fi8_[a-z0-9_]+":\s*&fi8\.([A-Za-z0-9]+)', block)
    for f in fields:
        assert f"fi8.{f}(" in doc, f
