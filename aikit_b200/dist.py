"""Row-sharded FlatI8 / FlatBinaryI8 across GPUs, one process per GPU.

The reference splits a corpus into contiguous shards and merges the
shard-local top-k sets by (score desc, index asc) (queryBatchSharded,
ann/backend.go:245-346; Flat.queryShards, ann/flat.go:188-229). Selection by
packed key decomposes exactly, so the multi-GPU form is: every rank scans its
contiguous row range [lo, hi) (global ids, so rank order is id order), the
M x k keys are all-gathered over NCCL, and every rank merges them on its
device (fi8_merge_keys_async).

FlatBinaryI8 needs the GLOBAL shortlist (the cand rows nearest in Hamming
distance over the whole corpus, ann/flat_binary_i8.go:105-106): every rank
prefilters its shard into sorted (-distance, id) keys, the keys are
all-gathered and merged into the global cand nearest, every rank reranks the
shortlist rows it holds, and the M x k results are merged again. That is the
reference's candidate set exactly.

torch.distributed carries the collectives (NCCL on GPUs, gloo on CPU for the
host-logic tests); the scans and merges are the library's kernels.
"""
from __future__ import annotations


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rank r holds rows [r*n//world, (r+1)*n//world): contiguous, in rank
    order, sizes differing by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return n * rank // world, n * (rank + 1) // world


class ShardedTopK:
    """TopKBatch over a row-sharded FlatI8: this rank's I8Index (built with
    id_base = its first global row) plus the cross-rank merge.

    overlap=True pipelines consecutive batches: the all-gather and merge of a
    batch run on a second (communication) stream while the next batch's scan
    runs on `stream`. The GEMM then leaves `free_sms` SMs to the collective's
    kernel (FI8_OPT_GEMM_CTAS), and two buffer slots alternate, so a result
    stays valid until the call after next. `wait()` orders `stream` after
    all communication issued so far."""

    def __init__(self, index, ctx, world: int, stream, group=None, overlap: bool = False, free_sms: int = 2):
        import torch
        self.ix, self.ctx, self.world, self.stream, self.group = index, ctx, world, stream, group
        self._torch = torch
        self._bufs = {}
        self.overlap = overlap and world > 1
        self.comm = None
        self._slot = 0
        self._done = [None, None]  # per slot: the event after its last all-gather and merge
        if self.overlap:
            self.comm = torch.cuda.Stream()
            index.set_gemm_ctas(max(1, ctx.sm_count() - free_sms))

    def _buffers(self, M: int, k: int, slot: int = 0):
        key = (M, k, slot)
        if key not in self._bufs:
            t = self._torch
            self._bufs[key] = (t.zeros((M, k), dtype=t.int64, device="cuda"),
                               t.zeros((self.world, M, k), dtype=t.int64, device="cuda"),
                               t.zeros((M, k), dtype=t.int64, device="cuda"))
        return self._bufs[key]

    def topk_async(self, d_q: int, M: int, k: int):
        """Device keys [M][k] of the global top-k (stream-ordered, no sync;
        with overlap, ordered on the communication stream: call wait() before
        reading them on `stream`). Every rank must call it with the same M
        and k."""
        import torch.distributed as dist
        if self.overlap:
            return self._topk_overlapped(d_q, M, k)
        local, gathered, merged = self._buffers(M, k)
        st = self.stream.cuda_stream
        self.ix.topk_async(d_q, M, k, local.data_ptr(), st)
        if self.world == 1:
            return local
        with self._torch.cuda.stream(self.stream):
            dist.all_gather_into_tensor(gathered.view(-1), local.view(-1), group=self.group)
        self.ctx.merge_keys_async(gathered.data_ptr(), self.world, M, k, merged.data_ptr(), st)
        return merged

    def _topk_overlapped(self, d_q: int, M: int, k: int):
        import torch.distributed as dist
        t = self._torch
        slot = self._slot
        self._slot ^= 1
        local, gathered, merged = self._buffers(M, k, slot)
        if self._done[slot] is not None:
            # this slot's previous all-gather has read `local` before the scan rewrites it
            self.stream.wait_event(self._done[slot])
        self.ix.topk_async(d_q, M, k, local.data_ptr(), self.stream.cuda_stream)
        scanned = t.cuda.Event()
        scanned.record(self.stream)
        self.comm.wait_event(scanned)
        with t.cuda.stream(self.comm):
            dist.all_gather_into_tensor(gathered.view(-1), local.view(-1), group=self.group)
        self.ctx.merge_keys_async(gathered.data_ptr(), self.world, M, k, merged.data_ptr(), self.comm.cuda_stream)
        done = t.cuda.Event()
        done.record(self.comm)
        self._done[slot] = done
        return merged

    def wait(self) -> None:
        """Order `stream` after every all-gather and merge issued so far."""
        if self.comm is not None:
            self.stream.wait_stream(self.comm)


class ShardedBinary:
    """FlatBinaryI8.Query over a row-sharded FlatBinaryI8 with the global
    shortlist (see the module doc)."""

    def __init__(self, index, ctx, world: int, stream, group=None):
        import torch
        self.ix, self.ctx, self.world, self.stream, self.group = index, ctx, world, stream, group
        self._torch = torch
        self._bufs = {}

    def _buffers(self, M: int, cand: int, k: int):
        key = (M, cand, k)
        if key not in self._bufs:
            t = self._torch
            z = lambda *s: t.zeros(s, dtype=t.int64, device="cuda")
            self._bufs[key] = (z(M, cand), z(self.world, M, cand), z(M, cand), z(M, k), z(self.world, M, k),
                               z(M, k))
        return self._bufs[key]

    def topk_async(self, d_q: int, M: int, k: int):
        """Device keys [M][k]: the reranked top-k of the global shortlist of
        cand = k * overquery rows (every rank calls it alike)."""
        import torch.distributed as dist
        cand = k * self.ix.overquery
        short, g_short, m_short, local, g_local, merged = self._buffers(M, cand, k)
        st = self.stream.cuda_stream
        if self.world == 1:
            self.ix.prefilter_async(d_q, M, cand, short.data_ptr(), st, sorted_keys=False)
            self.ix.rerank_async(d_q, M, short.data_ptr(), cand, k, local.data_ptr(), st)
            return local
        self.ix.prefilter_async(d_q, M, cand, short.data_ptr(), st, sorted_keys=True)
        with self._torch.cuda.stream(self.stream):
            dist.all_gather_into_tensor(g_short.view(-1), short.view(-1), group=self.group)
        self.ctx.merge_keys_async(g_short.data_ptr(), self.world, M, cand, m_short.data_ptr(), st)
        self.ix.rerank_async(d_q, M, m_short.data_ptr(), cand, k, local.data_ptr(), st)
        with self._torch.cuda.stream(self.stream):
            dist.all_gather_into_tensor(g_local.view(-1), local.view(-1), group=self.group)
        self.ctx.merge_keys_async(g_local.data_ptr(), self.world, M, k, merged.data_ptr(), st)
        return merged
