"""Build libchelis_cuda.so in-tree for sm_100a (nvcc cross-compiles; no GPU
needed).  The shared library is what travels to the GPU box and what
chelis_b200 loads.  One part compiles at run time: the per-chain FusedElem
kernels of csrc/fused_jit.cu, generated and compiled with NVRTC for sm_100a
at first use and cached per device; every other kernel is in this library."""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libchelis_cuda.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
    # IEEE division / square root and denormals; products and sums that must
    # match the C lane bit for bit use explicit __f*_rn intrinsics, which the
    # compiler never contracts into FMA.
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
    "-diag-suppress", "550",
]


def nvcc() -> str:
    path = os.environ.get("CHELIS_NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return path


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(ROOT, "include", "chelis_cuda.h"), __file__]
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-I", CSRC,
           os.path.join(CSRC, "libchelis_cuda.cu"), "-o", LIB + ".tmp", "-lcuda"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
