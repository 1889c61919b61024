"""Build recipe of the CUDA library: csrc/*.cu -> libneon_cuda.so, in-tree.

    python neon-runtime-beta-variation_b200/build.py [--verbose]

nvcc cross-compiles for sm_100a only (no GPU needed). The library links the
CUDA runtime statically and exports the C ABI of include/neon_cuda.h.
IEEE division, square root and denormals stay on (no --use_fast_math): the
Q8_0 activation quantiser must match the reference bit for bit.
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
INCLUDE = os.path.join(ROOT, "include")
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libneon_cuda.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
    "--expt-relaxed-constexpr",
]

SOURCES = ["neon_cuda.cu", "neon_decode.cu", "neon_comm.cu"]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return any(os.path.getmtime(p) > t for p in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    """Compile libneon_cuda.so if any source is newer than it; return its path."""
    if not force and not _stale():
        return LIB
    cmd = [_nvcc(), *NVCC_FLAGS, "-shared", "-I", INCLUDE, "-I", CSRC]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    cmd += ["-o", LIB + ".tmp"]
    subprocess.check_call(cmd)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
