"""A small, self-contained FlatI8 workload for profilers (ncu) and timing.

    python -m aikit_b200.profile_case --rows 2000000 --dim 768 --k 100 --batch 1 --reps 3

Builds a synthetic mixture corpus (the bench's recipe) of --rows rows on cuda:0
and runs --reps TopKBatch calls of --batch queries through the C ABI (device
buffers, one stream), then prints the per-call device time. Sized so that a
profiler capture of one launch ends in seconds while the corpus still exceeds L2.
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=2_000_000)
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--k", type=int, default=100)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--mode", choices=["topk", "score", "binary", "build", "probe"], default="topk")
    ap.add_argument("--recipe", choices=["mixture", "ties", "unit"], default="mixture",
                    help="corpus: C2/C3 mixture, C5 ties (codes in {-2..2}, scale 1/127), or iid unit rows")
    ap.add_argument("--over", type=int, default=100, help="binary mode: overquery (cand = k * over)")
    ap.add_argument("--tensor", type=int, default=0,
                    help="binary mode: prefilter batches of at least this many queries on the tensor cores")
    ap.add_argument("--pair", type=int, default=0, help="1: batched GEMM on CTA pairs (FI8_OPT_GEMM_PAIR)")
    ap.add_argument("--ctas", type=int, default=0, help="cap on the GEMM's CTAs (FI8_OPT_GEMM_CTAS; 0: every SM)")
    ap.add_argument("--trace", action="store_true",
                    help="also report per-kernel device time (torch.profiler / CUPTI) over the reps")
    a = ap.parse_args()

    import torch
    from aikit_b200 import synth
    from aikit_b200.ann import B200Backend

    be = B200Backend(0)
    if a.mode == "binary":
        return binary_case(a, be)
    if a.mode == "build":
        return build_case(a, be)
    if a.mode == "probe":
        out = {"mode": "probe"}
        for iters in (2000, 20000, 20000, 60000):
            ops, ms = be.ctx.probe_tensor_i8(iters)
            out.setdefault("runs", []).append({"iters": iters, "ms": round(ms, 3), "tops": round(ops / 1e12, 1)})
        print(json.dumps(out))
        return
    if a.recipe == "ties":
        r = synth.Recipe(synth.TIES, a.dim, seed=20265)
    elif a.recipe == "unit":
        r = synth.Recipe(synth.UNIT, a.dim, seed=20261)
    else:
        r = synth.Recipe(synth.MIXTURE, a.dim, seed=20260, ncl=1000, sigma=0.3)
    bq, bs = r.codes(a.rows)
    ix = be.NewI8Index(bq, bs, a.rows, a.dim)
    ix.set_gemm_pair(a.pair == 1)
    ix.set_gemm_ctas(a.ctas)
    Q = torch.from_numpy(r.queries(a.batch)).cuda()
    keys = torch.zeros((a.batch, a.k), dtype=torch.int64, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    times = []
    prof = None
    if a.trace and a.mode == "topk":  # per-launch device times from the library's events
        ix.set_kernel_timing(True)
    if a.trace and a.mode != "topk":
        from torch.profiler import ProfilerActivity, profile
        prof = profile(activities=[ProfilerActivity.CUDA])
        prof.__enter__()
    for _ in range(a.reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if a.mode == "topk":
            ix.topk_async(Q.data_ptr(), a.batch, a.k, keys.data_ptr(), stream.cuda_stream)
        else:
            dst = np.empty(a.batch * a.rows, np.float32)
            ix.ScoreBatch(Q.cpu().numpy(), dst)
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    ix.sync()
    kernels = None
    launch_log = None
    if a.trace and a.mode == "topk":
        log = ix.kernel_log()
        per = len(log) // max(a.reps, 1)
        launch_log = [(name, round(ms * 1e3, 1)) for name, ms, _ in log[-per:]]  # the last call
        kernels = {}
        for name, ms, _ in log[per:]:  # all but the first (cold) call
            t = kernels.setdefault(name, {"calls_per_rep": 0.0, "us_per_rep": 0.0})
            t["calls_per_rep"] += 1.0 / max(a.reps - 1, 1)
            t["us_per_rep"] += ms * 1e3 / max(a.reps - 1, 1)
    if prof is not None:
        prof.__exit__(None, None, None)
        agg = {}
        for ev in prof.events():
            if ev.device_type.name != "CUDA":
                continue
            name = next((k for k in ("scan_kernel", "gemm_kernel", "select_kernel", "quantize_kernel",
                                     "merge_keys_kernel", "Memcpy", "Memset") if k in ev.name), ev.name[:40])
            t = agg.setdefault(name, [0, 0.0])
            t[0] += 1
            t[1] += ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
        kernels = {k: {"calls_per_rep": v[0] / a.reps, "us_per_rep": v[1] / a.reps} for k, v in agg.items()}
    gbs = [a.rows * (a.dim + 4) / (t * 1e-3) / 1e9 for t in times]
    out = {"rows": a.rows, "dim": a.dim, "k": a.k, "batch": a.batch, "ms": times, "gbs_per_pass": gbs}
    if kernels is not None:
        out["kernels"] = kernels
    if launch_log is not None:
        out["last_call_launches_us"] = launch_log
    print(json.dumps(out))


def binary_case(a, be) -> None:
    """FlatBinaryI8 on a UNIT corpus (the C4 recipe): --reps batch queries of
    prefilter + rerank, device-resident, one stream."""
    import torch
    from aikit_b200 import synth
    r = synth.Recipe(synth.UNIT, a.dim, seed=20264)
    ctr = r.center(a.rows)
    bits, q8, sc = r.binary(a.rows, ctr)
    bix = be.NewBinaryI8Index(bits, bits.shape[1], ctr, q8, sc, a.rows, a.dim, a.over)
    del q8, sc
    if a.tensor:
        bix.set_tensor_prefilter(a.tensor)
    cand = a.k * a.over
    Q = torch.from_numpy(r.queries(a.batch)).cuda()
    short = torch.zeros((a.batch, cand), dtype=torch.int64, device="cuda")
    keys = torch.zeros((a.batch, a.k), dtype=torch.int64, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    times = []
    for rep in range(a.reps):
        if rep == 1:  # time kernels from the second (warm) call on
            bix.set_kernel_timing(a.trace)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        bix.prefilter_async(Q.data_ptr(), a.batch, cand, short.data_ptr(), stream.cuda_stream, sorted_keys=False)
        bix.rerank_async(Q.data_ptr(), a.batch, short.data_ptr(), cand, a.k, keys.data_ptr(), stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    bix.sync()
    gbs = [a.batch * a.rows * bits.shape[1] * 8 / (t * 1e-3) / 1e9 for t in times]
    out = {"mode": "binary", "rows": a.rows, "dim": a.dim, "k": a.k, "cand": cand, "batch": a.batch,
           "tensor_min_batch": a.tensor, "ms": times, "codes_gbs_per_pass": gbs,
           "queries_per_s": [a.batch / (t * 1e-3) for t in times]}
    if a.trace:  # per kernel class, from the library's CUDA events
        warm = max(a.reps - 1, 1)
        out["kernels"] = {k: {"launches_per_rep": v["launches"] / warm, "us_per_rep": v["ms"] * 1e3 / warm}
                          for k, v in bix.kernel_times().items()}
    print(json.dumps(out))


def build_case(a, be) -> None:
    """Device corpus builds from float rows: FlatI8 (quantize) and
    FlatBinaryI8 (quantize, float64 centre, sign codes), timed end to end
    from the host array (its upload included)."""
    import time
    from aikit_b200 import synth
    r = synth.Recipe(synth.MIXTURE, a.dim, seed=20262, ncl=1000, sigma=0.3)
    v = r.floats(a.rows)
    gb = v.nbytes / 1e9
    out = {"mode": "build", "rows": a.rows, "dim": a.dim, "float_gb": gb}
    for name, fn in (("flat_i8", lambda: be.NewI8IndexFromFloats(v)),
                     ("flat_binary_i8", lambda: be.NewBinaryI8IndexFromFloats(v))):
        times = []
        for _ in range(max(a.reps, 1)):
            t0 = time.perf_counter()
            ix = fn()
            times.append(time.perf_counter() - t0)
            ix.Close()
        best = min(times[1:] if len(times) > 1 else times)
        out[name] = {"s": times, "rows_per_s": a.rows / best, "float_gbs": gb / best}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
