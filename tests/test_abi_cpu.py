"""The C ABI surface without a GPU: the library loads, exports everything the
public header declares, and its host-side logic (the claim predicate, row
geometry, host repack, shard arithmetic) behaves like the reference's.

No call here launches a kernel or touches device memory.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from helpers import random_blocks


def test_library_exports_every_declared_symbol(G):
    L = G.lib()
    names = G.declared_symbols()
    assert len(names) >= 40, names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, f"declared in include/ggml-b200.h but not exported: {missing}"


def test_compat_entry_points_match_reference_names(G):
    """The eight compat entry points of include/xdna/ggml-xdna.h:156-165."""
    for n in ("ggml_backend_xdna_init", "ggml_backend_is_xdna", "ggml_backend_xdna_free",
              "ggml_backend_xdna_buffer_type", "ggml_backend_xdna_host_buffer_type",
              "ggml_backend_xdna_supports_op", "ggml_backend_xdna_compute_graph", "ggml_backend_xdna_reg"):
        assert n in G.declared_symbols()


def tensor_struct_layout(G):
    T = G.GgmlTensorXdna
    return {f[0]: getattr(T, f[0]).offset for f in T._fields_}, C.sizeof(T)


def test_tensor_struct_layout(G):
    """ggml_tensor_xdna as include/xdna/ggml-xdna.h:131-142 lays it out (LP64)."""
    off, size = tensor_struct_layout(G)
    assert off["type"] == 0 and off["ne"] == 8 and off["nb"] == 40 and off["op"] == 72
    assert off["op_params"] == 76 and off["flags"] == 140 and off["src"] == 144
    assert off["data"] == 224 and off["name"] == 232 and off["extra"] == 296 and size == 304


# ---------------------------------------------------------------- supports_op
def mm(G, wtype, K, N, M=1, xtype=None, nb1=None):
    w = G.tensor(wtype, [K, N], nb=[0, nb1] if nb1 is not None else None)
    x = G.tensor(G.F32 if xtype is None else xtype, [K, M])
    node = G.mul_mat_node(w, x, None, N, M)
    node._keep = (w, x)
    return node


def claims(G, node) -> bool:
    return bool(G.lib().ggml_backend_xdna_supports_op(None, C.byref(node)))


@pytest.mark.parametrize("t", [2, 11, 12, 13, 14, 18, 21, 22, 23])
def test_supports_claimed_formats(G, t):
    assert claims(G, mm(G, t, 4096, 4096))
    assert claims(G, mm(G, t, 2048, 11008))
    assert claims(G, mm(G, t, 4096, 32))


def test_supports_op_rejections(G):
    """src/ggml-xdna.cpp:95-147: MUL_MAT only, F32 src1, M == 1, N >= 32,
    N % 4 == 0, K a block multiple, nb[1] 0 or the packed row size."""
    assert claims(G, mm(G, G.Q4_0, 5120, 17408))
    assert not claims(G, mm(G, G.F32, 4096, 4096))               # unclaimed weight type
    assert not claims(G, mm(G, G.Q4_0, 4096, 4096, M=8))         # prefill batch
    assert not claims(G, mm(G, G.Q4_0, 4096, 4096, xtype=G.F16))  # non-F32 activations
    assert not claims(G, mm(G, G.Q4_0, 5121, 4096))              # K not a block multiple
    assert not claims(G, mm(G, G.Q4_K, 4096 + 32, 4096))         # K-quants need K % 256
    assert not claims(G, mm(G, G.Q4_0, 4096, 16))                # N < 32
    assert not claims(G, mm(G, G.Q4_0, 4096, 4098))              # N % 4 != 0
    assert claims(G, mm(G, G.Q4_0, 4096, 4096, nb1=4096 // 32 * 18))
    assert not claims(G, mm(G, G.Q4_0, 4096, 4096, nb1=4096 // 32 * 18 + 2))  # padded rows
    norm = G.tensor(G.F32, [4096, 1], op=G.GGML_OP_RMS_NORM)
    assert not claims(G, norm)
    assert not G.lib().ggml_backend_xdna_supports_op(None, None)


@pytest.mark.parametrize("t", [2, 11, 12, 13, 14, 18, 21, 22, 23])
def test_row_bytes(G, O, t):
    for K in (256, 2048, 11008 // 256 * 256):
        assert G.lib().b200_row_bytes(t, K) == O.row_bytes(t, K)
    assert G.lib().b200_row_bytes(t, 255) == 0


# ---------------------------------------------------------------- host repack
@pytest.mark.parametrize("t", [2, 11, 12, 13, 14, 18, 21, 22, 23])
@pytest.mark.parametrize("shape", [(64, 512), (40, 1024), (32, 256), (6, 256), (36, 512)])
def test_host_repack_round_trip(G, t, shape):
    N, K = shape
    raw = random_blocks(t, N, K, seed=N + K + t)
    packed = np.zeros_like(raw)
    back = np.zeros_like(raw)
    L = G.lib()
    assert L.b200_repack_host(t, raw.ctypes.data, packed.ctypes.data, N, K) == 0, G.last_error()
    assert L.b200_unpack_host(t, packed.ctypes.data, back.ctypes.data, N, K) == 0, G.last_error()
    np.testing.assert_array_equal(back, raw)
    # a permutation of the same bits within the same byte span (bytes move,
    # bit planes are transposed, 4-bit values re-paired): no padding needed
    assert packed.size == raw.size
    assert int(np.unpackbits(packed).sum()) == int(np.unpackbits(raw).sum())
    if N >= 8:
        assert not np.array_equal(packed, raw)


def test_host_repack_rejects_bad_shapes(G):
    raw = np.zeros(4096, np.uint8)
    L = G.lib()
    assert L.b200_repack_host(G.Q4_K, raw.ctypes.data, raw.ctypes.data, 4, 300) != 0  # K % 256
    assert L.b200_repack_host(99, raw.ctypes.data, raw.ctypes.data, 8, 256) != 0       # unknown type
    assert L.b200_repack_host(G.Q4_0, raw.ctypes.data, raw.ctypes.data, -1, 256) != 0  # negative N


# ---------------------------------------------------------------- sharding
def shard(G, n, world, rank):
    r0, nr = C.c_int64(), C.c_int64()
    rc = G.lib().ggml_backend_xdna_shard_rows(n, world, rank, C.byref(r0), C.byref(nr))
    return rc, r0.value, nr.value


def test_shard_rows_cover_exactly(G):
    for n, world in [(28672, 8), (128256, 8), (1024, 2), (8192, 4), (4096, 1)]:
        seen = []
        for r in range(world):
            rc, r0, nr = shard(G, n, world, r)
            assert rc == 0
            seen.append((r0, nr))
        assert seen[0][0] == 0 and sum(nr for _, nr in seen) == n
        assert all(a[0] + a[1] == b[0] for a, b in zip(seen, seen[1:]))


def test_shard_rows_rejects(G):
    assert shard(G, 1000, 3, 0)[0] != 0   # rows not divisible across ranks
    assert shard(G, 1024, 2, 2)[0] != 0   # rank out of range
    assert shard(G, 1024, 0, 0)[0] != 0
