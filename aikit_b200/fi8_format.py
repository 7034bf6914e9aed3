"""The FI8 v1 blob: FlatI8's persisted form (ann/flat_i8_persist.go:19-39).

    magic uint32 = 0x46493800 ("FI8\\0") | version uint32 = 1
    dim int32 | n int32
    codes:  n * dim int8, row-major
    scales: n * float32, little-endian

Validation follows flatI8Layout (ann/flat_i8_persist.go:165-194): bad magic,
other versions, negative shape scalars, n==0 xor dim==0, and any payload size
other than exactly n*dim + 4n are ErrFormat errors, never crashes. ``load``
returns a zero-copy view of the codes (the LoadFlatI8Mmap aliasing,
ann/flat_i8_mmap.go:157-180) and a copy of the scales.
"""
from __future__ import annotations

import mmap
import os
import struct

import numpy as np

MAGIC = 0x46493800
VERSION = 1


class FormatError(ValueError):
    """ann.ErrFormat (ann/format_errors.go:20)."""


def layout(data) -> tuple[int, int, int]:
    """(dim, n, codes_at) of a valid blob, else FormatError."""
    mv = memoryview(data)
    if len(mv) < 4:
        raise FormatError("ann: FlatI8 blob: truncated reading magic")
    if struct.unpack_from("<I", mv, 0)[0] != MAGIC:
        raise FormatError("ann: not a FlatI8 blob (bad magic)")
    if len(mv) < 8:
        raise FormatError("ann: FlatI8 blob: truncated reading version")
    v = struct.unpack_from("<I", mv, 4)[0]
    if v != VERSION:
        raise FormatError(f"ann: unsupported FlatI8 format version {v} (want {VERSION})")
    if len(mv) < 16:
        raise FormatError("ann: FlatI8 blob: truncated reading shape")
    dim, n = struct.unpack_from("<ii", mv, 8)
    if dim < 0:
        raise FormatError(f"ann: FlatI8 dim {dim} is negative")
    if n < 0:
        raise FormatError(f"ann: FlatI8 n {n} is negative")
    if (n == 0) != (dim == 0):
        raise FormatError(f"ann: FlatI8 inconsistent shape (n={n}, dim={dim}): both must be zero or both nonzero")
    want = n * dim + n * 4
    got = len(mv) - 16
    if want != got:
        raise FormatError(f"ann: FlatI8 payload size {got} != n*dim + n*4 = {want} (n={n} dim={dim})")
    return dim, n, 16


def load(data) -> tuple[np.ndarray, np.ndarray]:
    """LoadFlatI8: (codes [n, dim] int8 view of data, scales [n] float32 copy)."""
    dim, n, at = layout(data)
    codes = np.frombuffer(data, dtype=np.int8, count=n * dim, offset=at).reshape(n, dim)
    scales = np.frombuffer(data, dtype="<f4", count=n, offset=at + n * dim).astype(np.float32)
    return codes, scales


def load_mmap(path: str):
    """LoadFlatI8Mmap: codes alias a read-only mapping of the file."""
    with open(path, "rb") as fh:
        size = os.fstat(fh.fileno()).st_size
        if size == 0:
            raise FormatError("ann: FlatI8 blob: truncated reading magic")
        mm = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
    return load(mm)


# Rows per paging block: about 1 MiB of codes (pagedBlockRows,
# ann/flat_i8_mmap.go:46-56).
PAGED_BLOCK_BYTES = 1 << 20


def paged_block_rows(dim: int) -> int:
    return max(PAGED_BLOCK_BYTES // dim, 1) if dim > 0 else 1


def upload_paged(backend, path: str, block_rows: int = 0, id_base: int = 0):
    """EnableGPU for a paged index (LoadFlatI8MmapPaged, ann/flat_i8_mmap.go:
    75-102): map the blob read-only and walk its blocks in order, uploading
    each block's rows (fi8_index_upload_rows) and then releasing its pages
    from the process (MADV_DONTNEED on the clean, file-backed mapping), so a
    corpus larger than host RAM reaches the device with about one block
    resident at a time. Returns the device index (an aikit_b200.ann.I8Index)."""
    with open(path, "rb") as fh:
        if os.fstat(fh.fileno()).st_size == 0:
            raise FormatError("ann: FlatI8 blob: truncated reading magic")
        mm = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
    try:
        dim, n, at = layout(mm)
        if n == 0:
            raise FormatError("ann: FlatI8 blob holds no rows")
        rows = block_rows if block_rows > 0 else paged_block_rows(dim)
        codes = np.frombuffer(mm, dtype=np.int8, count=n * dim, offset=at)
        scales = np.frombuffer(mm, dtype="<f4", count=n, offset=at + n * dim)
        ix = backend.NewI8IndexEmpty(n, dim, id_base=id_base)
        page = mmap.PAGESIZE
        for r0 in range(0, n, rows):
            r1 = min(r0 + rows, n)
            ix.upload_rows(r0, codes[r0 * dim:r1 * dim], scales[r0:r1].astype(np.float32))
            # the block's whole pages are no longer needed on the host
            lo = -(-(at + r0 * dim) // page) * page
            hi = (at + r1 * dim) // page * page
            if hasattr(mmap, "MADV_DONTNEED") and hi > lo:
                mm.madvise(mmap.MADV_DONTNEED, lo, hi - lo)
        ix.upload_finish()
        del codes, scales
        return ix
    finally:
        try:
            mm.close()
        except BufferError:  # a view is still alive; the mapping closes with it
            pass


def dumps(codes: np.ndarray, scales: np.ndarray) -> bytes:
    """MarshalBinary (ann/flat_i8_persist.go:48-72)."""
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype="<f4")
    n = scales.shape[0]
    dim = codes.shape[1] if codes.ndim == 2 and n > 0 else 0
    return struct.pack("<IIii", MAGIC, VERSION, dim, n) + codes.tobytes() + scales.tobytes()
