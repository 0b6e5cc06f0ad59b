"""Build libggml-b200.so in-tree (nvcc, sm_100a) -- the product library.

    python build.py [--clean]

Outputs land next to this file: ``libggml-b200.so`` and ``_build/`` (object
files and the generated IQ table header).  The shared object links the CUDA
runtime statically so it can be dlopen'ed by a ggml host or ctypes without
any Python or torch runtime.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libggml-b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["gemv.cu", "gemv_mma.cu", "repack.cu", "quantize.cu"]
CXX_SOURCES = ["backend.cpp"]
HEADERS = ["formats.cuh", "gemv.cuh", "nccl_shim.h"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    tables = os.path.join(BUILD, "iq_tables.h")
    gen = os.path.join(CSRC, "gen_iq_tables.py")
    if _stale(tables, [gen]):
        subprocess.run([sys.executable, gen, tables], check=True)
    common = [os.path.join(CSRC, h) for h in HEADERS] + [tables, os.path.join(HERE, "..", "include", "ggml-b200.h")]
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", BUILD, "-I", CSRC,
                    "--expt-relaxed-constexpr"]
    objs = []
    for src in CU_SOURCES + CXX_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if _stale(o, [s] + common):
            cmd = [NVCC] + flags + (["-x", "cu"] if src.endswith(".cu") else []) + ["-c", s, "-o", o]
            if src.endswith(".cu"):
                cmd += ["-Xptxas", "-v"] if verbose else []
            subprocess.run(cmd, check=True)
    if _stale(LIB, objs):
        subprocess.run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-lrt", "-ldl", "-lpthread"],
                       check=True)
    return LIB


if __name__ == "__main__":
    if "--clean" in sys.argv:
        shutil.rmtree(BUILD, ignore_errors=True)
        if os.path.exists(LIB):
            os.remove(LIB)
    print(build(verbose="-v" in sys.argv))
