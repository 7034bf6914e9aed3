"""Multi-GPU parity (2 ranks, one process per GPU, NCCL): the row-sharded
FlatI8 top-k (aikit_b200.dist.ShardedTopK) and the sharded FlatBinaryI8 with
the global shortlist (ShardedBinary) equal the CPU oracle on the whole corpus,
including a corpus ordered against the query, whose shard-local batches drop
candidates and are redone on the device before the all-gather. Skipped on a
box with fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import oracle
    from aikit_b200 import synth
    from aikit_b200.ann import B200Backend, unpack_keys
    from aikit_b200.dist import ShardedBinary, ShardedTopK, shard_bounds

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    ok = True
    try:
        be = B200Backend(rank)
        stream = torch.cuda.Stream()
        torch.cuda.set_stream(stream)
        # FlatI8, batched (GEMM path) and single query (scan path)
        d, n, k = 256, 90001, 50
        r = synth.Recipe(synth.MIXTURE, d, seed=41, ncl=30, sigma=0.3)
        bq, bs = r.codes(n)
        lo, hi = shard_bounds(n, world, rank)
        ix = be.NewI8Index(bq[lo:hi], bs[lo:hi], hi - lo, d, id_base=lo)
        sh = ShardedTopK(ix, be.ctx, world, stream)
        for M in (16, 1):
            Q = r.queries(M, row0=M)
            qd = torch.from_numpy(Q).cuda()
            keys = sh.topk_async(qd.data_ptr(), M, k)
            stream.synchronize()
            ix.sync()
            gi, gs = unpack_keys(keys.cpu().numpy().view(np.uint64))
            if rank == 0:
                for m in range(M):
                    i, s = oracle.flat_i8_query(bq, bs, Q[m], k)
                    ok &= gi[m].tolist() == list(i) and gs[m].tobytes() == np.asarray(s, np.float32).tobytes()
        # pipelined batches: each all-gather + merge on a second stream beside
        # the next batch's scan, two result slots alternating
        sho = ShardedTopK(ix, be.ctx, world, stream, overlap=True)
        M = 24
        Qs = [r.queries(M, row0=100 + 50 * b) for b in range(3)]
        outs = []
        for b in range(3):
            qd = torch.from_numpy(Qs[b]).cuda()
            outs.append((qd, sho.topk_async(qd.data_ptr(), M, k)))
        sho.wait()
        stream.synchronize()
        ix.sync()
        for b in (1, 2):  # batch 0's slot was reused by batch 2
            gi, gs = unpack_keys(outs[b][1].cpu().numpy().view(np.uint64))
            if rank == 0:
                for m in range(0, M, 5):
                    i, s = oracle.flat_i8_query(bq, bs, Qs[b][m], k)
                    ok &= gi[m].tolist() == list(i) and gs[m].tobytes() == np.asarray(s, np.float32).tobytes()
        ix.Close()
        # a corpus ordered against the first query (every later row beats every
        # earlier one): each shard's batched top-k drops candidates and its
        # gated redo recomputes it before the all-gather reads the keys
        d, n, k = 64, 400_000, 20
        ra = synth.Recipe(synth.UNIT, d, seed=8)
        bq, bs = ra.codes(n)
        Q = ra.queries(6)
        aq, as_ = oracle.quantize_queries(Q[:1])
        order = np.argsort(oracle.w8a8(aq, as_, bq, bs)[0], kind="stable")
        bq, bs = np.ascontiguousarray(bq[order]), np.ascontiguousarray(bs[order])
        lo, hi = shard_bounds(n, world, rank)
        ix = be.NewI8Index(bq[lo:hi], bs[lo:hi], hi - lo, d, id_base=lo)
        for overlap in (False, True):
            sha = ShardedTopK(ix, be.ctx, world, stream, overlap=overlap)
            qd = torch.from_numpy(Q).cuda()
            keys = sha.topk_async(qd.data_ptr(), len(Q), k)
            sha.wait()
            stream.synchronize()
            ix.sync()
            gi, gs = unpack_keys(keys.cpu().numpy().view(np.uint64))
            if rank == 0:
                for m in range(len(Q)):
                    i, s = oracle.flat_i8_query(bq, bs, Q[m], k)
                    ok &= gi[m].tolist() == list(i) and gs[m].tobytes() == np.asarray(s, np.float32).tobytes()
        ix.Close()
        # FlatBinaryI8 with the global shortlist
        d, n, k, over = 512, 40000, 10, 30
        rb = synth.Recipe(synth.MIXTURE, d, seed=43, ncl=25, sigma=0.35)
        v = rb.floats(n)
        ctr = oracle.center(v)
        codes = oracle.pack_codes(v, ctr)
        bq, bs = oracle.quantize_rows(v)
        lo, hi = shard_bounds(n, world, rank)
        bix = be.NewBinaryI8Index(codes[lo:hi], codes.shape[1], ctr, bq[lo:hi], bs[lo:hi], hi - lo, d, over,
                                  id_base=lo)
        shb = ShardedBinary(bix, be.ctx, world, stream)
        M = 4
        Q = rb.queries(M)
        qd = torch.from_numpy(Q).cuda()
        keys = shb.topk_async(qd.data_ptr(), M, k)
        stream.synchronize()
        bix.sync()
        gi, gs = unpack_keys(keys.cpu().numpy().view(np.uint64))
        if rank == 0:
            for m in range(M):
                i, s = oracle.flat_binary_i8_query(codes, ctr, bq, bs, over, Q[m], k)
                ok &= gi[m].tolist() == list(i) and gs[m].tobytes() == np.asarray(s, np.float32).tobytes()
        bix.Close()
        results[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharded_parity():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: True, 1: True}
