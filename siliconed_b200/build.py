"""Builds the two libraries in-tree with nvcc for sm_100a (B200).

``python -m siliconed_b200.build`` (or ``__graft_entry__.build()``) compiles the CUDA sources under
``siliconed_b200/csrc`` into ``siliconed_b200/libsiliconed_cuda.so`` (the quantized linear stage) and
those under ``siliconed_b200/csrc/dit`` into ``siliconed_b200/libsiliconed_dit.so`` (the DiT blocks'
elementwise stages).  Both link the CUDA runtime statically; the first resolves the one driver entry
point it needs (cuTensorMapEncodeTiled) at run time, so they depend on nothing but the NVIDIA driver.
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
DIT_LIB = os.path.join(HERE, "libsiliconed_dit.so")
DIT_CSRC = os.path.join(CSRC, "dit")
DIT_SOURCES = ["sd_kernels.cu", "sd_attention.cu"]

SOURCES = ["sc_abi.cu", "sc_weight.cu", "sc_gemm.cu", "sc_gemm_pair.cu", "sc_gemm_bf16.cu", "sc_gemm_skinny.cu", "sc_gemm_skinny_sk.cu",
           "sc_gemv.cu", "sc_no_alloc.cu", "sc_rotate.cu", "sc_w8a8.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(lib: str, src_dir: str, header: str) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = [os.path.join(src_dir, f) for f in os.listdir(src_dir) if os.path.isfile(os.path.join(src_dir, f))]
    deps += [os.path.join(INCLUDE, header), os.path.join(CSRC, "sc_ptx.cuh"), __file__]
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(lib: str, src_dir: str, sources: list[str], verbose: bool) -> None:
    tmp = lib + ".tmp"
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-I", INCLUDE, "-I", src_dir, "-o", tmp]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(src_dir, s) for s in sources]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, lib)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles each library whose sources are newer than it; returns the linear stage's path."""
    if force or _stale(LIB, CSRC, "siliconed_cuda.h"):
        _compile(LIB, CSRC, SOURCES, verbose)
    if force or _stale(DIT_LIB, DIT_CSRC, "siliconed_dit.h"):
        _compile(DIT_LIB, DIT_CSRC, DIT_SOURCES, verbose)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
