"""Build libemberglass_cuda.so in-tree for sm_100a.

nvcc compiles the CUDA sources for `-gencode arch=compute_100a,code=sm_100a`
(cross-compiles without a GPU); g++ compiles the host quantiser/generator
with -ffp-contract=off so its arithmetic matches the reference's JS doubles
operation by operation.  Objects go to _build/ beside this file, the shared
library next to the package so it ships with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libemberglass_cuda.so")
INCLUDE = os.path.join(ROOT, "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = "/usr/bin/g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
           "-ccbin", CXX, "-I", INCLUDE, "-I", CSRC]
CXXFLAGS = ["-O3", "-std=c++17", "-fPIC", "-fopenmp", "-ffp-contract=off", "-march=x86-64-v3",
            "-I", INCLUDE, "-I", CSRC, "-I", "/usr/local/cuda/include"]

CU = ["eg_kernels.cu", "eg_batch.cu", "eg_tc.cu", "eg_prefill.cu", "eg_fused.cu", "eg_runtime.cu", "eg_noalloc.cu"]
CPP = ["eg_host.cpp", "eg_safetensors.cpp"]
HEADERS = ["eg_common.cuh", "eg_device.cuh", "eg_stream.cuh", "eg_tc.cuh", "eg_kernels.h", "eg_batch.h", "eg_prefill.h", "eg_fused.h",
           "eg_host.h"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(verbose: bool = False, extra_nvflags: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "emberglass.h")]
    objs = []
    for src in CU:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if _stale(o, [s, __file__] + hdrs):
            _run([NVCC, *ARCH, *NVFLAGS, *(extra_nvflags or []), "-c", s, "-o", o], verbose)
        objs.append(o)
    for src in CPP:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if _stale(o, [s, __file__] + hdrs):
            _run([CXX, *CXXFLAGS, "-c", s, "-o", o], verbose)
        objs.append(o)
    if _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-ccbin", CXX, "-o", LIB, *objs, "-Xcompiler", "-fopenmp",
              "-lgomp", "-Xlinker", "--no-undefined"], verbose)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
