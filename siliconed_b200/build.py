"""Builds libsiliconed_cuda.so in-tree with nvcc for sm_100a (B200).

``python -m siliconed_b200.build`` (or ``__graft_entry__.build()``) compiles every CUDA source under
``siliconed_b200/csrc`` into ``siliconed_b200/libsiliconed_cuda.so``.  The library links the CUDA
runtime statically and resolves the one driver entry point it needs (cuTensorMapEncodeTiled) at run
time, so it depends on nothing but the NVIDIA driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libsiliconed_cuda.so")

SOURCES = ["sc_abi.cu", "sc_weight.cu", "sc_gemm.cu", "sc_gemm_pair.cu", "sc_gemm_bf16.cu", "sc_gemv.cu",
           "sc_no_alloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, "siliconed_cuda.h"), __file__]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles the library if any source is newer than it; returns its path."""
    if not force and not _stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-I", INCLUDE, "-I", CSRC, "-o", tmp]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
