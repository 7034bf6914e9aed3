"""Record outputs of the reference's own CUDA kernels as a golden fixture.

Runs on a machine with a B200 and the built oracle/_ref/libref_anncuda.so (the
kernels of the reference's gpu/anncuda/gemv_w8a8.cu, compiled for sm_100a from
the reference source; oracle/ref_anncuda.py). It needs no reference source at
run time. For a few small seeded inputs it stores the int8 corpus rows and
scales, the int8 queries and scales (quantized as the reference's
quantizeRowInt8 does, gpu/anncuda/backend.go:270-298), and what the reference
kernels return: the W8A8 score matrix of launchBatch (backend.go:675-712) and
the top-k ids and scores of launchTopK (:468-510). tests/test_oracle.py checks
the CPU oracle against these reference-run outputs.

    python tests/golden/make_ref_gpu_golden.py OUT.npz
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from aikit_b200 import synth  # noqa: E402
import oracle  # noqa: E402
from oracle import ref_anncuda  # noqa: E402

# (name, recipe kind, n, dim, M, k): one case per reference launch form
CASES = [
    ("gemv_split", synth.MIXTURE, 9000, 32, 1, 10),    # gemv_w8a8; topk_split_r16 + topk_merge_r16
    ("byte_kpass", synth.MIXTURE, 3001, 100, 3, 100),  # batch8 byte path (dim % 4 != 0); topk_rows (k passes)
    ("ties_r64", synth.TIES, 4000, 64, 2, 50),         # batch8 over tied scores; topk_rows_r64
    ("wide_r32", synth.UNIT, 1500, 64, 20, 32),        # batch16, two query planes; topk_rows_r32
]


def main(out: str) -> None:
    import torch
    from aikit_b200.ann import Context
    sm = Context(0).sm_count()
    arrays = {}
    for name, kind, n, d, M, k in CASES:
        r = synth.Recipe(kind, d, seed=n + d + M, ncl=25, sigma=0.3) if kind == synth.MIXTURE else \
            synth.Recipe(kind, d, seed=n + d + M)
        bq, bs = r.codes(n)
        Q = r.queries(M)
        aq, as_ = oracle.quantize_queries(Q)
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        codes, scales, qi8, qs = dev(bq), dev(bs), dev(aq), dev(as_)
        scores = torch.empty((M, n), dtype=torch.float32, device="cuda")
        idx = torch.empty((M, k), dtype=torch.int32, device="cuda")
        val = torch.empty((M, k), dtype=torch.float32, device="cuda")
        ref = ref_anncuda.RefTopK(n, d, M, k, sm)
        ref.score(codes.data_ptr(), scales.data_ptr(), qi8.data_ptr(), qs.data_ptr(), scores.data_ptr())
        torch.cuda.synchronize()
        sc = scores.cpu().numpy().copy()
        ref.topk(scores.data_ptr(), idx.data_ptr(), val.data_ptr())
        torch.cuda.synchronize()
        ref.close()
        arrays.update({f"{name}/codes": bq, f"{name}/scales": bs, f"{name}/qi8": aq, f"{name}/qscale": as_,
                       f"{name}/k": np.int64(k), f"{name}/scores": sc,
                       f"{name}/idx": idx.cpu().numpy(), f"{name}/val": val.cpu().numpy()})
    np.savez_compressed(out, **arrays)
    print(f"wrote {out}: {len(CASES)} cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
