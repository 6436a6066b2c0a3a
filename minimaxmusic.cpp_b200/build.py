"""Builds libmm3fa.so (the C ABI of include/mm3fa.h) for sm_100a with nvcc.

Usage: python minimaxmusic.cpp_b200/build.py [--force] [--verbose]

The library is written next to this file (lib/libmm3fa.so) so it travels with the source
tree; it statically links the CUDA runtime and has no torch dependency.  NCCL is not linked:
the multi-GPU exchange loads libnccl.so.2 at run time (nccl.h supplies only the types).
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libmm3fa.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["mm3fa_abi.cu", "fa_decode.cu", "fa_decode_mma.cu", "fa_dense_sm100.cu", "fa_prologue.cu", "mm3fa_noalloc.cu",
           "mm3fa_exchange.cu"]
HEADERS = ["fa_common.cuh", "fa_decode.cuh", "fa_dense.cuh", "fa_prologue.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.sep not in c or os.path.exists(c)):
            return c
    return "nvcc"


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE, "mm3fa.h"), __file__]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    if not force and not ptxas_info and not _stale():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)

    def compile_one(src: str) -> str:
        obj = os.path.join(objdir, os.path.splitext(src)[0] + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-c", os.path.join(CSRC, src), "-o", obj]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        return obj

    # translation units compile in parallel; the link is one nvcc -shared step
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs, "-ldl"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print register / shared-memory use")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_info))


if __name__ == "__main__":
    main()
