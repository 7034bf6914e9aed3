"""Host-side mirror of the reference's device seam, over the C ABI.

The reference (Go) defines the seam in ann/backend.go:16-55:

    type Backend interface { NewI8Index(bq []int8, scales []float32, n, dim int) (I8Index, error); Name() string }
    type I8Index interface { Score(q, dst []float32) error; Close() error }
    type I8BatchIndex interface { ScoreBatch(queries [][]float32, dst []float32) error }
    type I8TopKIndex interface { TopKBatch(queries [][]float32, k int) ([][]Hit, error) }

and gpu/anncuda/backend.go implements it with CUDA. ``B200Backend`` and
``I8Index`` below keep those names, argument meanings and error behaviour (a
Go ``error`` becomes a raised ``Fi8Error``; a decline is ``DeclinedError``) so
the parity tests read like the reference's own. Every call goes to
libfi8_b200.so; nothing here computes a score.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Sequence

import numpy as np

from ._ffi import Fi8Error, check, lib


@dataclass(frozen=True)
class Hit:
    """ann.Hit (ann/flat.go:51-54): corpus index and float64-widened score."""

    Index: int
    Score: float


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def keep_bitmap(keep) -> np.ndarray:
    """A keep predicate as the ABI's bitmap: keep[id] truthy -> bit id%64 of
    word id/64 (uint64 words, little-endian bit order)."""
    bits = np.packbits(np.asarray(keep, dtype=bool), bitorder="little")
    pad = (-bits.size) % 8
    if pad:
        bits = np.concatenate([bits, np.zeros(pad, np.uint8)])
    return bits.view(np.uint64)


def device_count() -> int:
    n = C.c_int(0)
    check(lib().fi8_device_count(C.byref(n)))
    return n.value


class Context:
    """One CUDA device (fi8_ctx)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib().fi8_ctx_create(device, C.byref(h)))
        self._h = h
        self.device = device

    @property
    def handle(self):
        return self._h

    def sm_count(self) -> int:
        n = C.c_int(0)
        check(lib().fi8_ctx_sm_count(self._h, C.byref(n)))
        return n.value

    def probe_tensor_i8(self, iters: int = 20000) -> tuple[float, float]:
        """The int8 tensor-pipe rate (ops/s) and the probe's ms (fi8_probe_tensor_i8)."""
        ops = C.c_double(0.0)
        ms = C.c_double(0.0)
        check(lib().fi8_probe_tensor_i8(self._h, iters, C.byref(ops), C.byref(ms)))
        return ops.value, ms.value

    def merge_keys_async(self, d_in: int, nsrc: int, M: int, k: int, d_out: int, stream: int = 0) -> None:
        """Top k per query of nsrc device key lists [nsrc][M][k] -> [M][k]."""
        check(lib().fi8_merge_keys_async(self._h, C.c_void_p(d_in), nsrc, M, k, C.c_void_p(d_out),
                                         C.c_void_p(stream or None)))

    def close(self) -> None:
        if self._h:
            lib().fi8_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class B200Backend:
    """ann.Backend on one B200 (the role of cudaBackend, gpu/anncuda/backend.go:38)."""

    def __init__(self, device: int = 0):
        self.ctx = Context(device)

    def Name(self) -> str:
        return "cuda-b200"

    def NewI8Index(self, bq, scales, n: int, dim: int, id_base: int = 0) -> "I8Index":
        """gpu/anncuda/backend.go:124-154: copies codes and scales to the device."""
        bq = np.ascontiguousarray(bq, dtype=np.int8).reshape(-1)
        scales = _f32(scales).reshape(-1)
        if n <= 0 or dim <= 0:
            raise Fi8Error(1, f"gpu: empty int8 index (n={n} dim={dim})")
        if bq.shape[0] != n * dim or scales.shape[0] != n:
            raise Fi8Error(1, f"gpu: int8 index shape mismatch (bq {bq.shape[0]}, scales "
                              f"{scales.shape[0]}, n={n} dim={dim})")
        return I8Index(self.ctx, bq, scales, n, dim, id_base)

    def NewI8IndexFromFloats(self, vecs, id_base: int = 0) -> "I8Index":
        """NewFlatI8 on the device (fi8_index_create_f32): vecs [n, dim] float32
        rows, quantized on the GPU bit-identically to QuantizeRowInt8."""
        v = _f32(vecs)
        if v.ndim != 2 or v.shape[0] == 0 or v.shape[1] == 0:
            raise Fi8Error(1, f"gpu: empty int8 index (shape {v.shape})")
        h = C.c_void_p()
        check(lib().fi8_index_create_f32(self.ctx.handle, _p(v), v.shape[0], v.shape[1], id_base, C.byref(h)))
        return I8Index._adopt(self.ctx, h, v.shape[0], v.shape[1], id_base)

    def NewI8IndexEmpty(self, n: int, dim: int, id_base: int = 0) -> "I8Index":
        """An index of n all-zero rows to fill with I8Index.upload_rows
        (fi8_index_create_empty): the device path of a paged or streamed
        corpus, which never has to be resident on the host as a whole."""
        h = C.c_void_p()
        check(lib().fi8_index_create_empty(self.ctx.handle, n, dim, id_base, C.byref(h)))
        return I8Index._adopt(self.ctx, h, n, dim, id_base)

    def NewBinaryI8IndexFromFloats(self, vecs, overquery: int = 16, centered: bool = True, center=None,
                                   valid=None, id_base: int = 0) -> "BinaryI8Index":
        """newFlatBinaryI8 on the device (fi8_bin_index_create_f32): the FlatI8
        rows and the prefilter's centre and sign codes from [n, dim] float32
        rows. valid: optional per-row flags (False = a ragged row, left out of
        the centre with all-zero codes); center: optional given centre (a row
        shard of a larger corpus)."""
        v = _f32(vecs)
        if v.ndim != 2 or v.shape[0] == 0 or v.shape[1] == 0:
            raise Fi8Error(1, f"gpu: empty binary index (shape {v.shape})")
        n, dim = v.shape
        vd = None if valid is None else np.ascontiguousarray(valid, dtype=np.uint8).reshape(-1)
        if vd is not None and vd.shape[0] != n:
            raise Fi8Error(1, "gpu: valid flags length != n")
        ctr = None if center is None else _f32(center).reshape(-1)
        h = C.c_void_p()
        check(lib().fi8_bin_index_create_f32(self.ctx.handle, _p(v), _p(vd) if vd is not None else None, n, dim,
                                             overquery, 1 if centered else 0, _p(ctr) if ctr is not None else None,
                                             id_base, C.byref(h)))
        return BinaryI8Index._adopt(self.ctx, h, n, dim, (dim + 63) // 64, overquery, id_base)

    def NewBinaryI8IndexEmpty(self, n: int, dim: int, center, overquery: int = 16,
                              id_base: int = 0) -> "BinaryI8Index":
        """A FlatBinaryI8 shard of n all-zero rows to fill with
        BinaryI8Index.upload_rows (fi8_bin_index_create_empty): a corpus that
        is generated or read block by block never sits on the host whole.
        center: the prefilter's centre [dim] (None: uncentred)."""
        ctr = None if center is None else _f32(center).reshape(-1)
        if ctr is not None and ctr.shape[0] != dim:
            raise Fi8Error(1, f"gpu: center len {ctr.shape[0]} != dim {dim}")
        words = (dim + 63) // 64
        h = C.c_void_p()
        check(lib().fi8_bin_index_create_empty(self.ctx.handle, n, dim, words, _p(ctr) if ctr is not None else None,
                                               overquery, id_base, C.byref(h)))
        return BinaryI8Index._adopt(self.ctx, h, n, dim, words, overquery, id_base)

    def NewBinaryI8Index(self, codes, words: int, center, bq, scales, n: int, dim: int,
                         overquery: int = 16, id_base: int = 0) -> "BinaryI8Index":
        """A device FlatBinaryI8 shard from the prefilter's packed codes
        [n*words] uint64 and center [dim] (None: uncentred), plus the FlatI8
        rows bq [n*dim] int8 and scales [n] (ann/flat_binary_i8.go:57-62).
        overquery defaults to DefaultOverquery (ann/flat_binary_prefilter.go:51)."""
        codes = np.ascontiguousarray(codes, dtype=np.uint64).reshape(-1)
        bq = np.ascontiguousarray(bq, dtype=np.int8).reshape(-1)
        scales = _f32(scales).reshape(-1)
        if n <= 0 or dim <= 0:
            raise Fi8Error(1, f"gpu: empty binary index (n={n} dim={dim})")
        if codes.shape[0] != n * words or bq.shape[0] != n * dim or scales.shape[0] != n:
            raise Fi8Error(1, "gpu: binary index shape mismatch")
        if center is not None:
            center = _f32(center).reshape(-1)
            if center.shape[0] != dim:
                raise Fi8Error(1, f"gpu: center len {center.shape[0]} != dim {dim}")
        return BinaryI8Index(self.ctx, codes, words, center, bq, scales, n, dim, overquery, id_base)


class I8Index:
    """A device-resident FlatI8 shard: I8Index + I8BatchIndex + I8TopKIndex."""

    def __init__(self, ctx: Context, bq: np.ndarray, scales: np.ndarray, n: int, dim: int, id_base: int = 0):
        h = C.c_void_p()
        check(lib().fi8_index_create(ctx.handle, _p(bq), _p(scales), n, dim, id_base, C.byref(h)))
        self._h = h
        self.ctx = ctx
        self.n = n
        self.dim = dim
        self.id_base = id_base

    @classmethod
    def _adopt(cls, ctx: Context, h, n: int, dim: int, id_base: int) -> "I8Index":
        self = cls.__new__(cls)
        self._h, self.ctx, self.n, self.dim, self.id_base = h, ctx, n, dim, id_base
        return self

    def read_rows(self):
        """The index's int8 rows [n, dim] and scales [n], copied to the host."""
        bq = np.empty((self.n, self.dim), np.int8)
        sc = np.empty(self.n, np.float32)
        check(lib().fi8_index_read_rows(self._h, _p(bq), _p(sc)))
        return bq, sc

    def upload_rows(self, row0: int, codes, scales) -> None:
        """Copy rows [row0, row0 + len(scales)) to the device
        (fi8_index_upload_rows); the host arrays may be dropped on return."""
        c = np.ascontiguousarray(codes, dtype=np.int8).reshape(-1)
        s = _f32(scales).reshape(-1)
        rows = s.shape[0]
        if c.shape[0] != rows * self.dim:
            raise Fi8Error(1, f"fi8_index_upload_rows: {c.shape[0]} codes for {rows} rows of dim {self.dim}")
        check(lib().fi8_index_upload_rows(self._h, row0, _p(c), _p(s), rows))

    def upload_finish(self) -> None:
        """Wait for every upload_rows copy and free the staging buffers."""
        check(lib().fi8_index_upload_finish(self._h))

    # -- I8Index ---------------------------------------------------------
    def Score(self, q: Sequence[float], dst: np.ndarray) -> None:
        """Fills dst[j] with the W8A8 score of q against row j."""
        q = _f32(q)
        if q.shape[0] != self.dim:
            raise Fi8Error(1, f"gpu: query dim {q.shape[0]} != index dim {self.dim}")
        if dst.shape[0] != self.n or dst.dtype != np.float32 or not dst.flags.c_contiguous:
            raise Fi8Error(1, f"gpu: dst len {dst.shape[0]} != index n {self.n}")
        check(lib().fi8_score(self._h, _p(q), _p(dst)))

    def Close(self) -> None:
        if self._h:
            check(lib().fi8_index_destroy(self._h))
            self._h = None

    # -- I8BatchIndex ----------------------------------------------------
    def ScoreBatch(self, queries, dst: np.ndarray) -> None:
        Q = self._queries(queries)
        M = Q.shape[0]
        if dst.shape[0] != M * self.n or dst.dtype != np.float32 or not dst.flags.c_contiguous:
            raise Fi8Error(1, f"gpu: batch dst len {dst.shape[0]} != M*N {M * self.n}")
        if M == 0:
            return
        check(lib().fi8_score_batch(self._h, _p(Q), M, _p(dst)))

    # -- I8TopKIndex -----------------------------------------------------
    def TopKBatch(self, queries, k: int) -> list[list[Hit]]:
        idx, sc = self.topk_arrays(queries, k)
        out = []
        for m in range(idx.shape[0]):
            row = []
            for j in range(idx.shape[1]):
                i = int(idx[m, j])
                if i < 0:
                    break
                row.append(Hit(i, float(sc[m, j])))
            out.append(row)
        return out

    def topk_arrays(self, queries, k: int, keep=None):
        """TopKBatch as arrays: (int32 [M,k], float32 [M,k]), index -1 = empty.
        keep: optional boolean array over global ids (QueryFilter)."""
        Q = self._queries(queries)
        M = Q.shape[0]
        idx = np.empty((M, max(k, 0)), np.int32)
        sc = np.empty((M, max(k, 0)), np.float32)
        if M == 0:
            return idx, sc
        if keep is None:
            check(lib().fi8_topk_batch(self._h, _p(Q), M, k, _p(idx), _p(sc)))
        else:
            bm = keep_bitmap(keep)
            check(lib().fi8_topk_batch_keep(self._h, _p(Q), M, k, _p(bm), len(keep), _p(idx), _p(sc)))
        return idx, sc

    def QueryFilterBatch(self, queries, k: int, keep) -> list[list[Hit]]:
        """FlatI8.QueryFilter (ann/flat_i8.go:136) for a batch: keep[id]
        (a boolean array over global ids) selects the rows that may be hit."""
        idx, sc = self.topk_arrays(queries, k, keep=keep)
        return [[Hit(int(i), float(s)) for i, s in zip(idx[m], sc[m]) if i >= 0] for m in range(idx.shape[0])]

    def max_k(self) -> int:
        v = C.c_int32(0)
        check(lib().fi8_topk_max_k(self._h, C.byref(v)))
        return v.value

    # -- device-resident forms ------------------------------------------
    def topk_async(self, d_q: int, M: int, k: int, d_keys: int, stream: int = 0, d_keep: int = 0,
                   keep_nbits: int = 0) -> None:
        """Device-resident top-k; d_keep: optional device keep bitmap."""
        if d_keep:
            check(lib().fi8_topk_batch_async_keep(self._h, C.c_void_p(d_q), M, k, C.c_void_p(d_keep), keep_nbits,
                                                  C.c_void_p(d_keys), C.c_void_p(stream or None)))
        else:
            check(lib().fi8_topk_batch_async(self._h, C.c_void_p(d_q), M, k, C.c_void_p(d_keys),
                                             C.c_void_p(stream or None)))

    def topk1_noalloc(self, d_q: int, k: int, d_keys: int, stream: int = 0) -> None:
        """fi8_topk1_noalloc: one query's top-k with the library's fixed scratch
        (no device allocation on this call); device pointers, k <= 256."""
        check(lib().fi8_topk1_noalloc(self._h, C.c_void_p(d_q), k, C.c_void_p(d_keys),
                                      C.c_void_p(stream or None)))

    def sync(self) -> None:
        check(lib().fi8_index_sync(self._h))

    def last_launch_count(self) -> int:
        v = C.c_int32(0)
        check(lib().fi8_index_last_launch_count(self._h, C.byref(v)))
        return v.value

    def set_kernel_timing(self, on: bool) -> None:
        """Record a CUDA event pair around every kernel this index launches."""
        from ._ffi import FI8_OPT_KERNEL_TIMING
        check(lib().fi8_index_set_option(self._h, FI8_OPT_KERNEL_TIMING, 1 if on else 0))

    def kernel_times(self, reset: bool = True) -> dict:
        """Per kernel class: launches, summed device ms and algorithmic bytes of
        the launches timed since the last reset (waits for them to finish)."""
        from ._ffi import KERNEL_KINDS
        nk = len(KERNEL_KINDS)
        launches = (C.c_int64 * nk)()
        ms = (C.c_double * nk)()
        nbytes = (C.c_double * nk)()
        check(lib().fi8_index_kernel_times(self._h, launches, ms, nbytes, 1 if reset else 0))
        return {name: {"launches": int(launches[i]), "ms": float(ms[i]), "bytes": float(nbytes[i])}
                for i, name in enumerate(KERNEL_KINDS) if launches[i]}

    def kernel_log(self, cap: int = 4096) -> list:
        """The timed launches in order: (kernel class, device ms, algorithmic bytes)."""
        from ._ffi import KERNEL_KINDS
        n = C.c_int32(0)
        kinds = (C.c_int32 * cap)()
        ms = (C.c_double * cap)()
        nbytes = (C.c_double * cap)()
        check(lib().fi8_index_kernel_log(self._h, cap, C.byref(n), kinds, ms, nbytes))
        return [(KERNEL_KINDS[kinds[i]], ms[i], nbytes[i]) for i in range(n.value)]

    def set_gemm_min_batch(self, m: int) -> None:
        """Batches of at least m queries use the tensor-core GEMM path."""
        from ._ffi import FI8_OPT_GEMM_MIN_BATCH
        check(lib().fi8_index_set_option(self._h, FI8_OPT_GEMM_MIN_BATCH, m))

    def set_gemm_ctas(self, ctas: int) -> None:
        """Cap the batched GEMM's persistent CTAs (0: one per SM), leaving SMs
        free for work that overlaps it (an NCCL collective of another batch)."""
        from ._ffi import FI8_OPT_GEMM_CTAS
        check(lib().fi8_index_set_option(self._h, FI8_OPT_GEMM_CTAS, ctas))

    def set_gemm_pair(self, on: bool) -> None:
        """Run batches of more than 128 queries on CTA pairs (tcgen05
        cta_group::2) or on single CTAs (the default). Results are identical."""
        from ._ffi import FI8_OPT_GEMM_PAIR
        check(lib().fi8_index_set_option(self._h, FI8_OPT_GEMM_PAIR, 1 if on else 0))

    def _queries(self, queries) -> np.ndarray:
        if isinstance(queries, np.ndarray) and queries.ndim == 2:
            Q = _f32(queries)
            if Q.shape[1] != self.dim:
                raise Fi8Error(1, f"gpu: batch query dim {Q.shape[1]} != index dim {self.dim}")
            return Q
        rows = list(queries)
        for m, q in enumerate(rows):
            if len(q) != self.dim:
                raise Fi8Error(1, f"gpu: batch query {m} dim {len(q)} != index dim {self.dim}")
        if not rows:
            return np.empty((0, self.dim), np.float32)
        return _f32(np.stack([_f32(q) for q in rows]))

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass


class BinaryI8Index:
    """A device-resident FlatBinaryI8 shard (ann/flat_binary_i8.go): the sign-bit
    Hamming prefilter, then the int8 W8A8 rerank of its shortlist."""

    def __init__(self, ctx: Context, codes, words, center, bq, scales, n, dim, overquery, id_base):
        h = C.c_void_p()
        cptr = _p(center) if center is not None else None
        check(lib().fi8_bin_index_create(ctx.handle, _p(codes), words, cptr, _p(bq), _p(scales), n, dim,
                                         overquery, id_base, C.byref(h)))
        self._h = h
        ih = C.c_void_p()
        check(lib().fi8_bin_index_handle(h, C.byref(ih)))
        self._ih = ih
        self.ctx = ctx
        self.n = n
        self.dim = dim
        self.words = words
        self.overquery = max(int(overquery), 1)
        self.id_base = id_base

    @classmethod
    def _adopt(cls, ctx: Context, h, n, dim, words, overquery, id_base) -> "BinaryI8Index":
        self = cls.__new__(cls)
        self._h = h
        ih = C.c_void_p()
        check(lib().fi8_bin_index_handle(h, C.byref(ih)))
        self._ih = ih
        self.ctx, self.n, self.dim, self.words = ctx, n, dim, words
        self.overquery = max(int(overquery), 1)
        self.id_base = id_base
        return self

    def upload_rows(self, row0: int, codes, bq, scales) -> None:
        """Rows [row0, row0 + len(scales)): packed codes [rows, words] uint64,
        int8 rows [rows, dim] and scales (fi8_bin_upload_rows)."""
        codes = np.ascontiguousarray(codes, dtype=np.uint64)
        bq = np.ascontiguousarray(bq, dtype=np.int8)
        scales = _f32(scales).reshape(-1)
        rows = scales.shape[0]
        if codes.size != rows * self.words or bq.size != rows * self.dim:
            raise Fi8Error(1, "gpu: binary upload shape mismatch")
        check(lib().fi8_bin_upload_rows(self._h, row0, _p(codes), _p(bq), _p(scales), rows))

    def upload_finish(self) -> None:
        check(lib().fi8_bin_upload_finish(self._h))

    def center(self):
        """The prefilter's centre (float32 [dim]), or None when uncentred."""
        out = np.empty(self.dim, np.float32)
        has = C.c_int32(0)
        check(lib().fi8_bin_center(self._h, _p(out), C.byref(has)))
        return out if has.value else None

    def read_codes(self) -> np.ndarray:
        """The packed sign codes [n, words] uint64, copied to the host."""
        out = np.empty((self.n, self.words), np.uint64)
        check(lib().fi8_bin_read_codes(self._h, _p(out)))
        return out

    def read_rows(self):
        """The FlatI8 rows [n, dim] int8 and scales [n]."""
        bq = np.empty((self.n, self.dim), np.int8)
        sc = np.empty(self.n, np.float32)
        check(lib().fi8_index_read_rows(self._ih, _p(bq), _p(sc)))
        return bq, sc

    def set_tensor_prefilter(self, min_batch: int) -> None:
        """Prefilter batches of at least min_batch queries on the tensor cores
        (the codes unpacked to +1/-1 int8 rows on the device, n x dim bytes
        more HBM); 0 frees the rows and keeps every batch on the popcount
        pass. The shortlist is the same either way."""
        check(lib().fi8_bin_set_tensor_prefilter(self._h, int(min_batch)))

    def set_gemm_pair(self, on: bool) -> None:
        """The tensor-core prefilter's batches of more than 128 queries on CTA
        pairs or single CTAs (the default); the shortlist is the same."""
        from ._ffi import FI8_OPT_GEMM_PAIR
        check(lib().fi8_index_set_option(self._ih, FI8_OPT_GEMM_PAIR, 1 if on else 0))

    def Query(self, q, k: int) -> list[Hit]:
        """FlatBinaryI8.Query (flat_binary_i8.go:78) for one query."""
        return self.QueryBatch([q], k)[0]

    def QueryFilter(self, q, k: int, keep) -> list[Hit]:
        """FlatBinaryI8.QueryFilter (flat_binary_i8.go:83): keep[id] (boolean
        array over global ids) applies in the prefilter."""
        return self.QueryBatch([q], k, keep=keep)[0]

    def QueryBatch(self, queries, k: int, keep=None) -> list[list[Hit]]:
        idx, sc = self.topk_arrays(queries, k, keep=keep)
        return [[Hit(int(i), float(s)) for i, s in zip(idx[m], sc[m]) if i >= 0] for m in range(idx.shape[0])]

    def topk_arrays(self, queries, k: int, keep=None):
        Q = _f32(np.asarray(queries, dtype=np.float32).reshape(-1, self.dim))
        M = Q.shape[0]
        idx = np.empty((M, max(k, 0)), np.int32)
        sc = np.empty((M, max(k, 0)), np.float32)
        if M == 0:
            return idx, sc
        if keep is None:
            check(lib().fi8_bin_query_topk(self._h, _p(Q), M, k, _p(idx), _p(sc)))
        else:
            bm = keep_bitmap(keep)
            check(lib().fi8_bin_query_topk_keep(self._h, _p(Q), M, k, _p(bm), len(keep), _p(idx), _p(sc)))
        return idx, sc

    def prefilter_async(self, d_q: int, M: int, cand: int, d_keys: int, stream: int = 0,
                        sorted_keys: bool = True, d_keep: int = 0, keep_nbits: int = 0) -> None:
        """The shortlist keys (-distance, global id) into d_keys [M][cand];
        sorted_keys=False skips the sort (fine for the rerank, not a merge);
        d_keep: optional device keep bitmap over global ids."""
        check(lib().fi8_bin_prefilter_async_keep(self._h, C.c_void_p(d_q), M, cand, C.c_void_p(d_keep or None),
                                                 keep_nbits, C.c_void_p(d_keys), 1 if sorted_keys else 0,
                                                 C.c_void_p(stream or None)))

    def rerank_async(self, d_q: int, M: int, d_short: int, cand: int, k: int, d_keys: int,
                     stream: int = 0) -> None:
        check(lib().fi8_bin_rerank_async(self._h, C.c_void_p(d_q), M, C.c_void_p(d_short), cand, k,
                                         C.c_void_p(d_keys), C.c_void_p(stream or None)))

    def sync(self) -> None:
        check(lib().fi8_index_sync(self._ih))

    def last_launch_count(self) -> int:
        v = C.c_int32(0)
        check(lib().fi8_index_last_launch_count(self._ih, C.byref(v)))
        return v.value

    def set_kernel_timing(self, on: bool) -> None:
        from ._ffi import FI8_OPT_KERNEL_TIMING
        check(lib().fi8_index_set_option(self._ih, FI8_OPT_KERNEL_TIMING, 1 if on else 0))

    def kernel_times(self, reset: bool = True) -> dict:
        from ._ffi import KERNEL_KINDS
        nk = len(KERNEL_KINDS)
        launches = (C.c_int64 * nk)()
        ms = (C.c_double * nk)()
        nbytes = (C.c_double * nk)()
        check(lib().fi8_index_kernel_times(self._ih, launches, ms, nbytes, 1 if reset else 0))
        return {name: {"launches": int(launches[i]), "ms": float(ms[i]), "bytes": float(nbytes[i])}
                for i, name in enumerate(KERNEL_KINDS) if launches[i]}

    def Close(self) -> None:
        if self._h:
            check(lib().fi8_bin_index_destroy(self._h))
            self._h = None
            self._ih = None

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass


def unpack_keys(keys: np.ndarray):
    """Decode packed top-K keys (fi8_keys_unpack): (int32 idx, float32 score)."""
    keys = np.ascontiguousarray(keys, dtype=np.uint64)
    idx = np.empty(keys.shape, np.int32)
    sc = np.empty(keys.shape, np.float32)
    check(lib().fi8_keys_unpack(_p(keys), keys.size, _p(idx), _p(sc)))
    return idx, sc
