"""Builds libhct_b200.so in-tree with nvcc for sm_100a.

    python -m haagenti_b200.build [--verbose]

The library is the product: CUDA kernels (LZ4, INT4, spectral scatter,
tcgen05 IDCT contraction) plus the C++ host code behind include/hct_b200.h.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libhct_b200.so")
SOURCES = ["lz4_decode.cu", "int4_dequant.cu", "idct_gemm.cu", "fdct.cu", "hct_host.cu", "hct_encode.cpp",
           "hct_noalloc.cu", "holo.cu", "zstd_decode.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False, force: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(os.path.dirname(HERE), "include", "hct_b200.h")]
    if (not force and os.path.exists(OUT)
            and all(os.path.getmtime(OUT) >= os.path.getmtime(d) for d in deps)):
        return OUT
    cmd = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC,-fopenmp",
           "-Xcompiler", "-Wall", "-shared", "-o", OUT, *srcs, "-ldl", "-lgomp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
