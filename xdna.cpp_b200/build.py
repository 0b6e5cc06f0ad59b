"""Build libggml-b200.so in-tree (nvcc, sm_100a) -- the product library.

    python build.py [--clean]

Outputs land next to this file: ``libggml-b200.so`` and ``_build/`` (object
files and the generated IQ table header); with XDNA_LLAMA_CPP_DIR set to a
llama.cpp / ggml tree, also the ggml plugin ``libggml-b200-ggml.so``.  The shared object links the CUDA
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
    build_ggml_adapter()
    return LIB


GGML_ADAPTER = os.path.join(HERE, "libggml-b200-ggml.so")


def build_ggml_adapter() -> str | None:
    """The ggml plugin (ggml/ggml-b200-adapter.cpp -> libggml-b200-ggml.so,
    the library GGML_BACKEND_PATH names), built only when XDNA_LLAMA_CPP_DIR
    points at a llama.cpp / ggml source tree: its ggml/include and ggml/src
    supply ggml.h, ggml-backend.h and ggml-backend-impl.h.  ggml's own symbols
    resolve at load time from the ggml host process; libggml-b200.so is found
    next to the adapter."""
    tree = os.environ.get("XDNA_LLAMA_CPP_DIR")
    if not tree:
        return None
    inc = [os.path.join(tree, "ggml", "include"), os.path.join(tree, "ggml", "src")]
    if not os.path.exists(os.path.join(inc[0], "ggml-backend.h")) or not os.path.exists(
            os.path.join(inc[1], "ggml-backend-impl.h")):
        raise SystemExit(f"XDNA_LLAMA_CPP_DIR={tree}: ggml/include/ggml-backend.h or ggml/src/ggml-backend-impl.h "
                         "not found")
    src = os.path.join(HERE, "ggml", "ggml-b200-adapter.cpp")
    hdrs = [os.path.join(HERE, "..", "include", h) for h in ("ggml-b200.h", "ggml-b200-convert.h")]
    if _stale(GGML_ADAPTER, [src, LIB] + hdrs):
        cxx = os.environ.get("CXX", "g++")
        subprocess.run([cxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra"]
                       + sum((["-I", d] for d in inc + [os.path.join(HERE, "..", "include")]), [])
                       + [src, "-o", GGML_ADAPTER, "-L", HERE, "-lggml-b200", "-Wl,-rpath,$ORIGIN"], check=True)
    return GGML_ADAPTER


if __name__ == "__main__":
    if "--clean" in sys.argv:
        shutil.rmtree(BUILD, ignore_errors=True)
        if os.path.exists(LIB):
            os.remove(LIB)
    print(build(verbose="-v" in sys.argv))
