"""Regenerate the committed golden fixtures under tests/golden/.

Run where the reference tree is available, with its path as the only
argument; the outputs are committed so the tests never read the reference at
run time.

1. embedded_corpus_head.fi8 -- the first 512 rows of the reference's real
   Model2Vec FI8 v1 blob (examples/embedded-corpus/assets/index.bin, d=256,
   n=1747), re-serialised with aikit_b200.fi8_format.dumps; plus
   embedded_corpus_meta.json with the original header and SHA-256 digests of
   its code and scale sections.
2. retrieval_eval.npz -- the d=256 document/query embeddings and relevance
   lists of testdata/retrieval_eval.json (no texts), the fixture behind
   ann/retrieval_eval_test.go:118-131's recall floor.
3. fuzz_seed_flati8.bin -- the committed fuzz-corpus input
   ann/testdata/fuzz/FuzzLoadFlatI8/898c8926483c8b67 (16 bytes).
4. flat_i8_cases.json -- seeded synthetic FlatI8 queries with the oracle's
   (C restatement's) top-K, as regression goldens for the oracle and targets
   for the GPU parity tests.
"""
from __future__ import annotations

import ast
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from aikit_b200 import fi8_format, synth  # noqa: E402
import oracle  # noqa: E402


def main(ref: str) -> None:
    blob = open(os.path.join(ref, "examples/embedded-corpus/assets/index.bin"), "rb").read()
    dim, n, at = fi8_format.layout(blob)
    codes, scales = fi8_format.load(blob)
    head = 512
    open(os.path.join(HERE, "embedded_corpus_head.fi8"), "wb").write(
        fi8_format.dumps(codes[:head], scales[:head]))
    meta = {
        "source": "examples/embedded-corpus/assets/index.bin",
        "dim": dim, "n": n, "bytes": len(blob), "head_rows": head,
        "codes_sha256": hashlib.sha256(blob[at:at + n * dim]).hexdigest(),
        "scales_sha256": hashlib.sha256(blob[at + n * dim:]).hexdigest(),
    }
    json.dump(meta, open(os.path.join(HERE, "embedded_corpus_meta.json"), "w"), indent=1)

    fx = json.load(open(os.path.join(ref, "testdata/retrieval_eval.json")))
    docs = np.array([d["emb"] for d in fx["docs"]], np.float32)
    qs = np.array([q["emb"] for q in fx["queries"]], np.float32)
    rel = np.full((len(fx["queries"]), max(len(q["relevant"]) for q in fx["queries"])), -1, np.int32)
    for i, q in enumerate(fx["queries"]):
        rel[i, :len(q["relevant"])] = q["relevant"]
    np.savez_compressed(os.path.join(HERE, "retrieval_eval.npz"), dim=fx["dim"], docs=docs,
                        queries=qs, relevant=rel)

    seed_txt = open(os.path.join(ref, "ann/testdata/fuzz/FuzzLoadFlatI8/898c8926483c8b67")).read()
    lit = seed_txt.strip().splitlines()[1]
    assert lit.startswith("[]byte(") and lit.endswith(")")
    raw = ast.literal_eval("b" + lit[len("[]byte("):-1])
    open(os.path.join(HERE, "fuzz_seed_flati8.bin"), "wb").write(raw)

    cases = {}
    for name, kind, n_, d_, k_, nq, extra in [
        ("unit_n3000_d96_k10", synth.UNIT, 3000, 96, 10, 8, {}),
        ("unit_n5000_d100_k25", synth.UNIT, 5000, 100, 25, 6, {}),
        ("mix_n20000_d768_k100", synth.MIXTURE, 20000, 768, 100, 4, dict(ncl=50, sigma=0.3)),
        ("ties_n8000_d64_k300", synth.TIES, 8000, 64, 300, 4, {}),
    ]:
        r = synth.Recipe(kind, d_, seed=11, **extra)
        bq, sc = r.codes(n_)
        Q = r.queries(nq)
        idx = np.full((nq, k_), -1, np.int64)
        score = np.zeros((nq, k_), np.float64)
        for m in range(nq):
            i, s = oracle.flat_i8_query(bq, sc, Q[m], k_)
            idx[m, :len(i)] = i
            score[m, :len(s)] = s
        cases[name] = dict(kind=kind, n=n_, d=d_, k=k_, nq=nq, seed=11,
                           ncl=extra.get("ncl", 0), sigma=extra.get("sigma", 0.0),
                           codes_sha256=hashlib.sha256(bq.tobytes()).hexdigest(),
                           idx=idx.tolist(), score=score.tolist())
    json.dump(cases, open(os.path.join(HERE, "flat_i8_cases.json"), "w"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference tree>")
    main(sys.argv[1])
