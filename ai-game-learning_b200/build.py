"""Build libpbgb200.so in-tree for sm_100a (nvcc cross-compiles without a GPU).

    python ai-game-learning_b200/build.py [--force]

Sources whose results must follow the reference's operation order one
rounding at a time (state machine, policy composition, RNG, showdown) are
compiled with ``-fmad=false``; the HBM-bound loss and optimizer kernels keep
fused multiply-adds, and the loss flushes denormals (``-ftz=true``).
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "pbg_b200")
LIB = os.path.join(OUT_DIR, "libpbgb200.so")
BUILD = os.path.join(HERE, "_build")

EXACT = ["common.cu", "poker.cu", "policy.cu", "showdown.cu", "completion.cu", "targets.cu", "posterior.cu", "branching.cu",
         "incidence.cu"]
FAST = ["loss.cu", "learner.cu", "mlp.cu", "model_backward.cu", "adam.cu", "collective.cu", "gemm.cu", "attention.cu", "layernorm.cu", "folded.cu", "eigh.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "pbgb200.h"))
    objects = []
    for name in EXACT + FAST:
        src = os.path.join(CSRC, name)
        obj = os.path.join(BUILD, name.replace(".cu", ".o"))
        objects.append(obj)
        if not force and not _stale(obj, [src, *headers, __file__]):
            continue
        flags = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-rdc=false",
                 "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-c", src, "-o", obj]
        if name in EXACT:
            flags.insert(5, "-fmad=false")
        if name == "loss.cu":
            flags.insert(5, "-ftz=true")
        if verbose:
            flags.insert(5, "-Xptxas=-v")
        subprocess.run(flags, check=True)
    if force or _stale(LIB, objects):
        subprocess.run([nvcc(), *ARCH, "-shared", "-o", LIB, *objects, "-lcudart"], check=True)
    return LIB


if __name__ == "__main__":
    p = argparse.ArgumentParser()
    p.add_argument("--force", action="store_true")
    p.add_argument("--verbose", action="store_true", help="print ptxas register/spill usage")
    a = p.parse_args()
    print(build(a.force, a.verbose))
    sys.exit(0)
