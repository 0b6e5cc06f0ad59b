"""Python binding of libggml-b200.so (the B200 decode-GEMV backend).

A thin ctypes mirror of include/ggml-b200.h: the reference's compat C ABI
(``ggml_backend_xdna_*``), the buffer interface and the launcher layer.  There
is no fallback: if the shared object is missing, importing the symbols raises.

Device memory and streams may come from anywhere (torch, cuda-python); the
launcher calls take raw device addresses and a cudaStream_t as an integer.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from functools import lru_cache

HERE = os.path.dirname(os.path.abspath(__file__))
# XDNA_B200_LIB selects another build of the library (the role GGML_BACKEND_PATH
# plays for a ggml host); the default is the in-tree build.
LIB_PATH = os.environ.get("XDNA_B200_LIB") or os.path.join(HERE, "libggml-b200.so")
HEADER = os.path.join(HERE, "..", "include", "ggml-b200.h")

# ggml type ids
F32, F16 = 0, 1
Q4_0, Q3_K, Q4_K, Q5_K, Q6_K = 2, 11, 12, 13, 14
IQ3_XXS, IQ3_S, IQ2_S, IQ4_XS = 18, 21, 22, 23
CLAIMED = {"Q4_0": Q4_0, "Q3_K": Q3_K, "Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K,
           "IQ3_XXS": IQ3_XXS, "IQ3_S": IQ3_S, "IQ2_S": IQ2_S, "IQ4_XS": IQ4_XS}
TYPE_NAME = {v: k for k, v in CLAIMED.items()}
BLOCK = {Q4_0: (32, 18), Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
         IQ3_XXS: (256, 98), IQ3_S: (256, 110), IQ2_S: (256, 82), IQ4_XS: (256, 136)}

# compat-ABI op ids (reference standalone enumeration: MUL_MAT = 18)
GGML_OP_NONE, GGML_OP_RMS_NORM, GGML_OP_MUL_MAT = 0, 15, 18


class GgmlTensorXdna(C.Structure):
    pass


GgmlTensorXdna._fields_ = [
    ("type", C.c_int),
    ("ne", C.c_int64 * 4),
    ("nb", C.c_size_t * 4),
    ("op", C.c_uint32),
    ("op_params", C.c_int32 * 16),
    ("flags", C.c_int32),
    ("src", C.POINTER(GgmlTensorXdna) * 10),
    ("data", C.c_void_p),
    ("name", C.c_char * 64),
    ("extra", C.c_void_p),
]


def row_bytes(t: int, K: int) -> int:
    bv, bb = BLOCK[t]
    return (K // bv) * bb


def tensor(type_: int, ne, data=None, nb=None, name: str = "", op: int = GGML_OP_NONE) -> GgmlTensorXdna:
    t = GgmlTensorXdna()
    t.type = type_
    ne = list(ne) + [1] * (4 - len(ne))
    for i in range(4):
        t.ne[i] = ne[i]
    if nb is not None:
        for i, v in enumerate(nb):
            t.nb[i] = v
    t.op = op
    t.data = data
    t.name = name.encode()[:63]
    return t


def mul_mat_node(w: GgmlTensorXdna, x: GgmlTensorXdna, y_data, N: int, M: int = 1, name: str = "mm") -> GgmlTensorXdna:
    node = tensor(F32, [N, M, 1, 1], data=y_data, name=name, op=GGML_OP_MUL_MAT)
    node.src[0] = C.pointer(w)
    node.src[1] = C.pointer(x)
    return node


def declared_symbols() -> list[str]:
    """Function names declared in include/ggml-b200.h."""
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(ggml_backend_\w+|b200_\w+)\s*\(", txt)))


@lru_cache(maxsize=None)
def lib() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python xdna.cpp_b200/build.py`")
    L = C.CDLL(LIB_PATH)
    vp, sz, i64, b = C.c_void_p, C.c_size_t, C.c_int64, C.c_bool
    tp = C.POINTER(GgmlTensorXdna)
    sig = {
        "ggml_backend_xdna_init": (vp, [sz]),
        "ggml_backend_is_xdna": (b, [vp]),
        "ggml_backend_xdna_free": (None, [vp]),
        "ggml_backend_xdna_buffer_type": (vp, [sz]),
        "ggml_backend_xdna_host_buffer_type": (vp, []),
        "ggml_backend_xdna_supports_op": (b, [vp, tp]),
        "ggml_backend_xdna_compute_graph": (b, [vp, C.POINTER(tp), sz]),
        "ggml_backend_xdna_reg": (vp, []),
        "ggml_backend_xdna_last_error": (C.c_char_p, []),
        "ggml_backend_xdna_buft_name": (C.c_char_p, [vp]),
        "ggml_backend_xdna_buft_alloc_buffer": (vp, [vp, sz]),
        "ggml_backend_xdna_buft_get_alignment": (sz, [vp]),
        "ggml_backend_xdna_buft_get_alloc_size": (sz, [vp, tp]),
        "ggml_backend_xdna_buft_is_host": (b, [vp]),
        "ggml_backend_xdna_buffer_free": (None, [vp]),
        "ggml_backend_xdna_buffer_get_base": (vp, [vp]),
        "ggml_backend_xdna_buffer_get_size": (sz, [vp]),
        "ggml_backend_xdna_buffer_set_tensor": (b, [vp, tp, vp, sz, sz]),
        "ggml_backend_xdna_buffer_get_tensor": (b, [vp, tp, vp, sz, sz]),
        "ggml_backend_xdna_buffer_memset_tensor": (b, [vp, tp, C.c_uint8, sz, sz]),
        "ggml_backend_xdna_buffer_clear": (b, [vp, C.c_uint8]),
        "ggml_backend_xdna_buffer_set_tensor_device": (b, [vp, tp, vp, sz, sz]),
        "ggml_backend_xdna_buffer_cpy_tensor": (b, [tp, tp]),
        "ggml_backend_xdna_get_stream": (vp, [vp]),
        "ggml_backend_xdna_synchronize": (None, [vp]),
        "ggml_backend_xdna_nccl_unique_id": (C.c_int, [C.c_char_p]),
        "ggml_backend_xdna_init_sharded": (vp, [sz, C.c_int, C.c_int, C.c_char_p]),
        "ggml_backend_xdna_shard_rows": (C.c_int, [i64, C.c_int, C.c_int, C.POINTER(i64), C.POINTER(i64)]),
        "ggml_backend_xdna_get_device_memory": (None, [sz, C.POINTER(sz), C.POINTER(sz)]),
        "ggml_backend_xdna_get_device_count": (sz, []),
        "b200_gemv": (C.c_int, [C.c_int, vp, vp, vp, i64, i64, vp, C.c_int]),
        "b200_gemv_noalloc": (C.c_int, [C.c_int, vp, vp, vp, i64, i64, vp]),
        "b200_gemv_multi": (C.c_int, [C.c_int, C.POINTER(vp), C.POINTER(vp), C.POINTER(i64), C.c_int, vp, i64, vp,
                                      C.c_int]),
        "b200_gemv_error": (C.c_int, [C.POINTER(C.c_int)]),
        "b200_repack": (C.c_int, [C.c_int, vp, vp, i64, i64, vp]),
        "b200_unpack": (C.c_int, [C.c_int, vp, vp, i64, i64, vp]),
        "b200_bf16_to_f32": (C.c_int, [vp, vp, i64, vp]),
        "b200_gemv_bf16": (C.c_int, [C.c_int, vp, vp, vp, i64, i64, vp, C.c_int]),
        "b200_fill_normal": (C.c_int, [vp, i64, C.c_uint64, C.c_float, vp]),
        "b200_quantize": (C.c_int, [C.c_int, vp, vp, i64, i64, vp]),
        "b200_repack_host": (C.c_int, [C.c_int, vp, vp, i64, i64]),
        "b200_unpack_host": (C.c_int, [C.c_int, vp, vp, i64, i64]),
        "b200_row_bytes": (sz, [C.c_int, i64]),
        "b200_gemv_smem_bytes": (sz, [C.c_int, i64]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return L


def last_error() -> str:
    return lib().ggml_backend_xdna_last_error().decode()


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        raise RuntimeError(f"{what}: {last_error()} (rc={rc})")


# ------------------------------------------------------------------ helpers
def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().ggml_backend_xdna_nccl_unique_id(buf), "nccl_unique_id")
    return buf.raw


def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    r0, nr = C.c_int64(), C.c_int64()
    check(lib().ggml_backend_xdna_shard_rows(n, world, rank, C.byref(r0), C.byref(nr)), "shard_rows")
    return r0.value, nr.value


class Backend:
    """RAII wrapper of a compat-ABI backend handle on one CUDA device
    (row-sharded over `world` ranks when an NCCL unique id is given)."""

    def __init__(self, dev: int = 0, world: int = 1, rank: int = 0, nccl_id: bytes | None = None):
        if nccl_id is None:
            self.h = lib().ggml_backend_xdna_init(dev)
        else:
            self.h = lib().ggml_backend_xdna_init_sharded(dev, world, rank, nccl_id)
        if not self.h:
            raise RuntimeError(f"ggml_backend_xdna_init(dev={dev}, world={world}, rank={rank}) failed: {last_error()}")
        self.dev, self.world, self.rank = dev, world, rank

    def supports_op(self, node: GgmlTensorXdna) -> bool:
        return bool(lib().ggml_backend_xdna_supports_op(self.h, C.byref(node)))

    def compute(self, nodes) -> bool:
        arr = (C.POINTER(GgmlTensorXdna) * len(nodes))(*[C.pointer(n) for n in nodes])
        return bool(lib().ggml_backend_xdna_compute_graph(self.h, arr, len(nodes)))

    def synchronize(self) -> None:
        lib().ggml_backend_xdna_synchronize(self.h)

    @property
    def stream(self) -> int:
        return lib().ggml_backend_xdna_get_stream(self.h) or 0

    def close(self) -> None:
        if self.h:
            lib().ggml_backend_xdna_free(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Buffer:
    """A buffer of the device (HBM) or host buffer type."""

    def __init__(self, size: int, dev: int = 0, host: bool = False):
        L = lib()
        self.buft = L.ggml_backend_xdna_host_buffer_type() if host else L.ggml_backend_xdna_buffer_type(dev)
        self.h = L.ggml_backend_xdna_buft_alloc_buffer(self.buft, size)
        if not self.h:
            raise RuntimeError(f"alloc_buffer({size}) failed: {last_error()}")
        self.base = L.ggml_backend_xdna_buffer_get_base(self.h)
        self.size = size
        self._next = 0

    def alloc(self, t: GgmlTensorXdna) -> GgmlTensorXdna:
        """Place tensor t at the next aligned offset (a trivial ggml-alloc)."""
        L = lib()
        align = L.ggml_backend_xdna_buft_get_alignment(self.buft)
        n = L.ggml_backend_xdna_buft_get_alloc_size(self.buft, C.byref(t))
        off = (self._next + align - 1) // align * align
        if off + n > self.size:
            raise MemoryError("buffer full")
        t.data = self.base + off
        self._next = off + n
        return t

    @staticmethod
    def copy(src: GgmlTensorXdna, dst: GgmlTensorXdna) -> None:
        if not lib().ggml_backend_xdna_buffer_cpy_tensor(C.byref(src), C.byref(dst)):
            raise RuntimeError(f"cpy_tensor failed: {last_error()}")

    def set_device(self, t: GgmlTensorXdna, dev_ptr: int, offset: int, size: int) -> None:
        if not lib().ggml_backend_xdna_buffer_set_tensor_device(self.h, C.byref(t), dev_ptr, offset, size):
            raise RuntimeError(f"set_tensor_device failed: {last_error()}")

    def set(self, t: GgmlTensorXdna, host_ptr: int, offset: int, size: int) -> None:
        if not lib().ggml_backend_xdna_buffer_set_tensor(self.h, C.byref(t), host_ptr, offset, size):
            raise RuntimeError(f"set_tensor failed: {last_error()}")

    def get(self, t: GgmlTensorXdna, host_ptr: int, offset: int, size: int) -> None:
        if not lib().ggml_backend_xdna_buffer_get_tensor(self.h, C.byref(t), host_ptr, offset, size):
            raise RuntimeError(f"get_tensor failed: {last_error()}")

    def memset(self, t: GgmlTensorXdna, value: int, offset: int, size: int) -> None:
        if not lib().ggml_backend_xdna_buffer_memset_tensor(self.h, C.byref(t), value, offset, size):
            raise RuntimeError(f"memset_tensor failed: {last_error()}")

    def clear(self, value: int) -> None:
        if not lib().ggml_backend_xdna_buffer_clear(self.h, value):
            raise RuntimeError(f"clear failed: {last_error()}")

    def free(self) -> None:
        if self.h:
            lib().ggml_backend_xdna_buffer_free(self.h)
            self.h = None
