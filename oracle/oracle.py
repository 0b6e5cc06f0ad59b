"""ctypes front end to the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Loaded by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg.
The product library (xdna.cpp_b200) never imports this module.

* ``_build/liboracle.so`` -- quant_oracle.c, the plain-C restatement of the
  reference's scalar path for all nine formats.
* ``_ref/libxdna_ref.so`` -- the reference's own CPU sources compiled in place
  by oracle/Makefile (present only where the reference tree was available at
  build time; the built .so travels with the repository snapshot).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from functools import lru_cache

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libxdna_ref.so")

# ggml type ids (reference include/xdna/ggml-xdna.h:19-48)
Q4_0, Q3_K, Q4_K, Q5_K, Q6_K, IQ3_XXS, IQ3_S, IQ2_S, IQ4_XS = 2, 11, 12, 13, 14, 18, 21, 22, 23
TYPES = {"Q4_0": Q4_0, "Q3_K": Q3_K, "Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K,
         "IQ3_XXS": IQ3_XXS, "IQ3_S": IQ3_S, "IQ2_S": IQ2_S, "IQ4_XS": IQ4_XS}
TYPE_NAMES = {v: k for k, v in TYPES.items()}
# types with an in-repo reference implementation (include/xdna/kquants.h, src/xdna-q4-0-reference.cpp)
REF_TYPES = (Q4_0, Q3_K, Q4_K, Q5_K, Q6_K, IQ3_S, IQ4_XS)

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")


def build(ref_dir: str | None = None) -> None:
    """Compile the oracle (and oracle/_ref when the reference tree is given,
    by argument or by the XDNA_REFERENCE_DIR environment variable)."""
    ref_dir = ref_dir if ref_dir is not None else os.environ.get("XDNA_REFERENCE_DIR", "")
    subprocess.run(["make", "-C", HERE, f"REF_DIR={ref_dir}", "all"], check=True,
                   stdout=subprocess.DEVNULL)


@lru_cache(maxsize=None)
def lib() -> C.CDLL:
    if not os.path.exists(ORACLE_SO):
        build()
    L = C.CDLL(ORACLE_SO)
    L.oracle_block_values.argtypes = [C.c_int]
    L.oracle_block_bytes.argtypes = [C.c_int]
    L.oracle_row_bytes.argtypes = [C.c_int, C.c_int64]
    L.oracle_row_bytes.restype = C.c_size_t
    L.oracle_fp16_to_f32.argtypes = [C.c_uint16]
    L.oracle_fp16_to_f32.restype = C.c_float
    L.oracle_f32_to_fp16.argtypes = [C.c_float]
    L.oracle_f32_to_fp16.restype = C.c_uint16
    L.oracle_bf16_to_f32.argtypes = [C.c_uint16]
    L.oracle_bf16_to_f32.restype = C.c_float
    L.oracle_f32_to_bf16.argtypes = [C.c_float]
    L.oracle_f32_to_bf16.restype = C.c_uint16
    L.oracle_dequantize_row.argtypes = [C.c_int, _u8p, C.c_int64, _f32p]
    L.oracle_gemv.argtypes = [C.c_int, _u8p, C.c_int64, C.c_int64, _f32p, _f32p, C.c_int]
    L.oracle_gemv_q4_0_bf16.argtypes = [_u8p, C.c_int64, C.c_int64, _u16p, _f32p, C.c_int]
    L.oracle_quantize.argtypes = [C.c_int, _f32p, C.c_int64, C.c_int64, _u8p, C.c_int]
    return L


def ref_available() -> bool:
    return os.path.exists(REF_SO)


@lru_cache(maxsize=None)
def ref() -> C.CDLL:
    if not ref_available():
        raise FileNotFoundError(f"{REF_SO} not built (reference tree absent at build time)")
    R = C.CDLL(REF_SO)
    R.ref_last_error.restype = C.c_char_p
    R.ref_q4_0_dequantize_row.argtypes = [_u8p, C.c_size_t, C.c_size_t, _f32p]
    R.ref_q4_0_gemv_f32.argtypes = [_u8p, C.c_size_t, C.c_size_t, C.c_size_t, _f32p, _f32p]
    R.ref_q4_0_gemv_bf16.argtypes = [_u8p, C.c_size_t, C.c_size_t, C.c_size_t, _u16p, _f32p]
    R.ref_fp16_to_f32.argtypes = [C.c_uint16]
    R.ref_fp16_to_f32.restype = C.c_float
    R.ref_kquant_dequantize_row.argtypes = [C.c_int, _u8p, C.c_int64, _f32p]
    R.ref_kquant_gemv.argtypes = [C.c_int, _u8p, C.c_size_t, C.c_size_t, _f32p, _f32p]
    R.ref_iq3s_grid.argtypes = [np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")]
    R.ref_kvalues_iq4nl.argtypes = [np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")]
    R.ref_bytes_per_row.argtypes = [C.c_int, C.c_size_t]
    R.ref_bytes_per_row.restype = C.c_size_t
    R.ref_engine_create.argtypes = [C.c_size_t]
    R.ref_engine_create.restype = C.c_void_p
    R.ref_engine_destroy.argtypes = [C.c_void_p]
    R.ref_engine_hardware_ready.argtypes = [C.c_void_p]
    R.ref_engine_run.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_size_t,
                                 C.c_size_t, C.c_void_p, C.c_void_p]
    R.ref_engine_run_bf16.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_size_t,
                                      C.c_size_t, C.c_void_p, C.c_void_p]
    R.ref_evaluate.argtypes = [_f32p, _f32p, C.c_size_t, C.c_size_t, C.c_double,
                               np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")]
    R.ref_tile_partition.argtypes = [C.c_size_t, C.c_size_t, C.c_size_t,
                                     C.POINTER(C.c_size_t), C.POINTER(C.c_size_t),
                                     np.ctypeslib.ndpointer(dtype=np.uintp, flags="C_CONTIGUOUS"),
                                     C.c_size_t]
    R.ref_q4_prepack_dequantize.argtypes = [_u8p, C.c_size_t, C.c_size_t, C.c_size_t, _f32p]
    return R


def _ref_check(rc: int) -> None:
    if rc != 0:
        raise ValueError(ref().ref_last_error().decode())


# ---------------------------------------------------------------- geometry
def block_values(t: int) -> int:
    return lib().oracle_block_values(t)


def block_bytes(t: int) -> int:
    return lib().oracle_block_bytes(t)


def row_bytes(t: int, K: int) -> int:
    return lib().oracle_row_bytes(t, K)


# ---------------------------------------------------------------- oracle
def quantize(t: int, x: np.ndarray, nthreads: int = 8) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    N, K = x.shape
    out = np.zeros(N * row_bytes(t, K), dtype=np.uint8)
    if lib().oracle_quantize(t, x, N, K, out, nthreads) != 0:
        raise ValueError("oracle_quantize failed")
    return out


def dequantize_row(t: int, row: np.ndarray, K: int) -> np.ndarray:
    out = np.empty(K, dtype=np.float32)
    if lib().oracle_dequantize_row(t, np.ascontiguousarray(row, dtype=np.uint8), K, out) != 0:
        raise ValueError("oracle_dequantize_row failed")
    return out


def gemv(t: int, w: np.ndarray, N: int, K: int, x: np.ndarray, nthreads: int = 8) -> np.ndarray:
    y = np.empty(N, dtype=np.float32)
    rc = lib().oracle_gemv(t, np.ascontiguousarray(w, dtype=np.uint8), N, K,
                           np.ascontiguousarray(x, dtype=np.float32), y, nthreads)
    if rc != 0:
        raise ValueError(f"oracle_gemv failed ({rc})")
    return y


def gemv_q4_0_bf16(w: np.ndarray, N: int, K: int, x_bf16: np.ndarray, nthreads: int = 8) -> np.ndarray:
    y = np.empty(N, dtype=np.float32)
    rc = lib().oracle_gemv_q4_0_bf16(np.ascontiguousarray(w, dtype=np.uint8), N, K,
                                     np.ascontiguousarray(x_bf16, dtype=np.uint16), y, nthreads)
    if rc != 0:
        raise ValueError("oracle_gemv_q4_0_bf16 failed")
    return y


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Reference float_to_bf16 (src/xdna-q4-0-reference.cpp:146-154), vectorised."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFFFFFF
    return (u >> 16).astype(np.uint16)


# ---------------------------------------------------------------- reference
def ref_gemv(t: int, w: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    """The reference's own scalar GEMV (q4_0::gemv_f32 or gemv_*_ref)."""
    y = np.empty(N, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if t == Q4_0:
        _ref_check(ref().ref_q4_0_gemv_f32(w, w.size, N, K, x, y))
    else:
        _ref_check(ref().ref_kquant_gemv(t, w, N, K, x, y))
    return y


def ref_dequantize_row(t: int, row: np.ndarray, K: int) -> np.ndarray:
    out = np.empty(K, dtype=np.float32)
    row = np.ascontiguousarray(row, dtype=np.uint8)
    if t == Q4_0:
        _ref_check(ref().ref_q4_0_dequantize_row(row, row.size, K, out))
    else:
        _ref_check(ref().ref_kquant_dequantize_row(t, row, K, out))
    return out


class RefEngine:
    """The reference's CPU GEMV engine (XdnaGemvEngine without XRT): AVX2 +
    OpenMP, src/xdna-gemv-engine.cpp:1817-1992."""

    def __init__(self, crossover_n: int = 256):
        self.R = ref()
        self.h = self.R.ref_engine_create(crossover_n)
        if not self.h:
            raise RuntimeError(self.R.ref_last_error().decode())

    def run(self, t: int, w: np.ndarray, N: int, K: int, x: np.ndarray, y: np.ndarray) -> None:
        rc = self.R.ref_engine_run(self.h, t, w.ctypes.data, w.nbytes, N, K, x.ctypes.data, y.ctypes.data)
        _ref_check(rc)

    def close(self) -> None:
        if self.h:
            self.R.ref_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- metrics
def stats(actual: np.ndarray, reference: np.ndarray) -> dict:
    """cos / maxabs / relL2 in float64, as tests/test-gemv-accuracy.cpp:34-57."""
    a = actual.astype(np.float64)
    r = reference.astype(np.float64)
    d = a - r
    na, nr = float(np.sqrt((a * a).sum())), float(np.sqrt((r * r).sum()))
    if na == 0.0 and nr == 0.0:
        cos = 1.0
    else:
        cos = float((a * r).sum() / (na * nr)) if na * nr > 1e-12 else 0.0
    maxabs = float(np.abs(d).max()) if d.size else 0.0
    rel_l2 = float(np.sqrt((d * d).sum()) / nr) if nr > 1e-12 else 0.0
    ymax = float(np.abs(r).max()) if r.size else 0.0
    return {"cos": cos, "maxabs": maxabs, "rel_l2": rel_l2, "maxabs_rel": maxabs / ymax if ymax > 0 else maxabs}
