"""Build recipe for the native libraries of aikit_b200.

* ``lib/libfi8_b200.so`` -- the CUDA library behind ``include/fi8.h``, compiled
  for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``).
* ``lib/libfi8_synth.so`` -- the seeded synthetic-corpus generator (host C).

Built in-tree so the shared objects travel with the repository snapshot.
Run ``python -m aikit_b200.build`` (``--ptxas`` prints register/spill
reports).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")

CUDA_SOURCES = ["fi8_api.cu", "fi8_scan.cu", "fi8_gemm.cu", "fi8_binary.cu", "fi8_build.cu"]
CUDA_HEADERS = ["fi8_device.cuh", "fi8_scan.cuh", "fi8_select.cuh", "fi8_gemm.cuh", "fi8_binary.cuh", "fi8_build.cuh", "fi8_stage.h"]
SYNTH_SOURCES = ["synth.c"]

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB_FI8 = os.path.join(LIBDIR, "libfi8_b200.so")
LIB_SYNTH = os.path.join(LIBDIR, "libfi8_synth.so")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build failed: " + " ".join(cmd))
    if os.environ.get("FI8_BUILD_VERBOSE"):
        sys.stderr.write(r.stdout + r.stderr)


def build_fi8(force: bool = False, ptxas: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in CUDA_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in CUDA_HEADERS] + [os.path.join(ROOT, "include", "fi8.h")]
    if not (force or ptxas) and not _stale(LIB_FI8, deps):
        return LIB_FI8
    os.makedirs(LIBDIR, exist_ok=True)
    cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
           "-shared", "-o", LIB_FI8, *srcs, "-lcudart"]
    if ptxas:
        cmd.insert(1, "-Xptxas=-v")
        os.environ["FI8_BUILD_VERBOSE"] = "1"
    _run(cmd)
    return LIB_FI8


def build_synth(force: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in SYNTH_SOURCES]
    if not force and not _stale(LIB_SYNTH, srcs):
        return LIB_SYNTH
    os.makedirs(LIBDIR, exist_ok=True)
    _run(["gcc", "-O3", "-ffp-contract=off", "-fno-fast-math", "-fno-math-errno", "-msse4.1", "-fPIC",
          "-shared", "-pthread",
          "-o", LIB_SYNTH, *srcs, "-lm"])
    return LIB_SYNTH


def build_all(force: bool = False) -> None:
    build_fi8(force)
    build_synth(force)


if __name__ == "__main__":
    build_fi8(force="--force" in sys.argv, ptxas="--ptxas" in sys.argv)
    build_synth(force="--force" in sys.argv)
    print(LIB_FI8)
    print(LIB_SYNTH)
