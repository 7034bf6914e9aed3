"""Multi-process (gloo, world size 2 and 3, CPU) tests of the row-sharded
decomposition the multi-GPU path uses (aikit_b200/dist.py): contiguous shards
in rank order with global ids, an all-gather of every rank's M x k packed keys,
and a top-k of the union -- the merge rule of queryBatchSharded / hitCmp
(ann/backend.go:262-277, ann/flat.go:298). The per-rank answers come from the
CPU oracle, so the test exercises the host-side plumbing and the merge rule,
not a GPU. FlatBinaryI8's global shortlist is checked the same way: per-shard
prefilterHist keys (-distance, id), merged, equal the full corpus's.
"""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import oracle
    from aikit_b200 import synth
    from aikit_b200.dist import shard_bounds
    from parity_util import make_keys, top_keys

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        # FlatI8 top-k, with a shard smaller than k when world is 3
        r = synth.Recipe(synth.MIXTURE, 96, seed=17, ncl=12, sigma=0.3)
        n, k, M = 4003 if world == 2 else 60, 25, 3
        bq, bs = r.codes(n)
        Q = r.queries(M)
        lo, hi = shard_bounds(n, world, rank)
        local = np.zeros((M, k), np.uint64)
        for m in range(M):
            i, s = oracle.flat_i8_query(bq[lo:hi], bs[lo:hi], Q[m], k)
            local[m] = top_keys(make_keys(np.asarray(i) + lo, np.asarray(s, np.float32)), k)
        gathered = torch.zeros((world, M, k), dtype=torch.int64)
        dist.all_gather_into_tensor(gathered.view(-1), torch.from_numpy(local.view(np.int64)).reshape(-1))
        g = gathered.numpy().view(np.uint64)
        ok = True
        for m in range(M):
            merged = top_keys(g[:, m, :], k)
            i, s = oracle.flat_i8_query(bq, bs, Q[m], k)
            want = top_keys(make_keys(i, np.asarray(s, np.float32)), k)
            ok &= merged.tobytes() == want.tobytes()

        # FlatBinaryI8: the global shortlist from per-shard prefilters
        v = synth.Recipe(synth.UNIT, 192, seed=5).floats(3001)
        ctr = oracle.center(v)
        codes = oracle.pack_codes(v, ctr)
        cand = 90
        lo, hi = shard_bounds(len(v), world, rank)
        qc = oracle.pack_row(v[7] + 0.01, ctr)
        d_loc = oracle.hamming_rows(qc, codes[lo:hi]).astype(np.int64)
        keys = make_keys(np.arange(lo, hi), -d_loc.astype(np.float32))
        mine = top_keys(keys, cand)
        gk = torch.zeros((world, cand), dtype=torch.int64)
        dist.all_gather_into_tensor(gk.view(-1), torch.from_numpy(mine.view(np.int64)))
        merged = top_keys(gk.numpy().view(np.uint64), cand)
        got_ids = sorted(int(0x7FFFFFFF - ((x >> np.uint64(1)) & np.uint64(0x7FFFFFFF))) for x in merged if x)
        want_ids = oracle.prefilter_hist(qc, codes, 192, cand).tolist()
        ok &= got_ids == want_ids
        results[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_merge_gloo(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {r: True for r in range(world)}


def test_shard_bounds():
    from aikit_b200.dist import shard_bounds
    for n in (0, 1, 7, 100, 10_000_000):
        for world in (1, 2, 3, 8):
            b = [shard_bounds(n, world, r) for r in range(world)]
            assert b[0][0] == 0 and b[-1][1] == n
            assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
            assert max(h - l for l, h in b) - min(h - l for l, h in b) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def test_host_key_layout_matches_library():
    """The test-side key packing decodes through the library's own
    fi8_keys_unpack (host code, no GPU) to the same index and score bits."""
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from aikit_b200.ann import unpack_keys
    from parity_util import make_keys
    rng = np.random.default_rng(3)
    idx = rng.integers(0, 2**31 - 1, 1000)
    sc = rng.standard_normal(1000).astype(np.float32)
    sc[:4] = [0.0, -0.0, np.inf, -np.inf]
    gi, gs = unpack_keys(make_keys(idx, sc))
    assert gi.tolist() == idx.tolist()
    assert gs.tobytes() == sc.tobytes()
    order = np.argsort(make_keys(idx, sc))[::-1]
    pairs = sorted(zip((-sc.astype(np.float64)).tolist(), idx.tolist()))
    assert [int(idx[o]) for o in order] == [p[1] for p in pairs]
