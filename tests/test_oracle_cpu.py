"""The CPU oracle, pinned: golden fixtures, the reference's known answers, and
(where oracle/_ref was built) the reference's own code live.

The oracle (oracle/quant_oracle.c) restates the reference's scalar GEMV in the
reference's float order, so for the seven formats the reference implements it
must agree bit for bit; IQ3_XXS and IQ2_S are pinned to the gguf 0.19.0
dequantiser with a float64 dot (the reference has no code for them).
"""
from __future__ import annotations

import glob
import os

import numpy as np
import pytest

from helpers import COS_MIN, MAXABS_REL

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "gemv_*.npz")))


def load(path):
    z = np.load(path)
    return {k: z[k] for k in z.files}


def test_all_formats_have_fixtures(O):
    names = {os.path.basename(p)[5:-4] for p in FIXTURES}
    assert names == set(O.TYPES), names


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: os.path.basename(p)[5:-4])
def test_oracle_matches_golden(O, path):
    f = load(path)
    t, N, K = int(f["type"]), int(f["N"]), int(f["K"])
    y = O.gemv(t, f["w"], N, K, f["x"], nthreads=1)
    deq0 = O.dequantize_row(t, f["w"][: O.row_bytes(t, K)], K)
    if t in O.REF_TYPES:
        # same arithmetic, same order as the reference: bit-exact
        np.testing.assert_array_equal(deq0, f["deq0"])
        np.testing.assert_array_equal(y, f["y"])
    else:
        np.testing.assert_allclose(deq0, f["deq0"], rtol=1e-6, atol=0)
        s = O.stats(y, f["y"])
        assert s["cos"] >= COS_MIN and s["maxabs_rel"] <= MAXABS_REL, s


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: os.path.basename(p)[5:-4])
def test_oracle_thread_count_does_not_change_results(O, path):
    f = load(path)
    t, N, K = int(f["type"]), int(f["N"]), int(f["K"])
    np.testing.assert_array_equal(O.gemv(t, f["w"], N, K, f["x"], nthreads=1),
                                  O.gemv(t, f["w"], N, K, f["x"], nthreads=4))


# ---------------------------------------------------------------- known answers
def edge_block() -> np.ndarray:
    """tests/test-q4-0-reference.cpp:49-54: d = 1.0, low nibbles 0..15, high 15..0."""
    return np.array([0x00, 0x3C, 0xF0, 0xE1, 0xD2, 0xC3, 0xB4, 0xA5, 0x96,
                     0x87, 0x78, 0x69, 0x5A, 0x4B, 0x3C, 0x2D, 0x1E, 0x0F], dtype=np.uint8)


def test_kat_q4_0_edge_block(O):
    deq = O.dequantize_row(O.Q4_0, edge_block(), 32)
    np.testing.assert_array_equal(deq[:16], np.arange(16) - 8.0)
    np.testing.assert_array_equal(deq[16:], 7.0 - np.arange(16))
    x = np.arange(1, 33, dtype=np.float32)
    assert O.gemv(O.Q4_0, edge_block(), 1, 32, x)[0] == -264.0
    assert O.gemv_q4_0_bf16(edge_block(), 1, 32, O.f32_to_bf16(x))[0] == -264.0


def test_kat_q4_0_two_rows(O):
    """tests/test-q4-0-reference.cpp:129-143,193-210: rows of +1 (d=1) and -1 (d=0.5)."""
    m = np.zeros(36, dtype=np.uint8)
    m[0:2] = [0x00, 0x3C]
    m[2:18] = 0x99
    m[18:20] = [0x00, 0x38]
    m[20:36] = 0x77
    x = np.arange(1, 33, dtype=np.float32)
    np.testing.assert_array_equal(O.gemv(O.Q4_0, m, 2, 32, x), [528.0, -264.0])
    np.testing.assert_array_equal(O.gemv_q4_0_bf16(m, 2, 32, O.f32_to_bf16(x)), [528.0, -264.0])


def uniform_q4_0(N, K, d_bits):
    w = np.zeros((N, K // 32, 18), dtype=np.uint8)
    w[:, :, 0] = d_bits & 0xFF
    w[:, :, 1] = d_bits >> 8
    w[:, :, 2:] = 0x99
    return w.reshape(-1)


def test_kat_compute_graph_128(O):
    """tests/test-backend.cpp:59-97: 128 x 256, d = 1, q - 8 = 1, x = 0.5 -> 128.0."""
    y = O.gemv(O.Q4_0, uniform_q4_0(128, 256, 0x3C00), 128, 256, np.full(256, 0.5, np.float32))
    np.testing.assert_array_equal(y, np.full(128, 128.0, np.float32))


def test_kat_uniform_scale(O):
    """tests/test-gemv-accuracy.cpp:127-153: 256 x 256, d = 0.5, x = 0.25 -> 32.0."""
    y = O.gemv(O.Q4_0, uniform_q4_0(256, 256, 0x3800), 256, 256, np.full(256, 0.25, np.float32))
    np.testing.assert_array_equal(y, np.full(256, 32.0, np.float32))


@pytest.mark.parametrize("name", ["Q4_0", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ3_XXS", "IQ3_S", "IQ2_S", "IQ4_XS"])
def test_zero_activation_gives_exact_zero(O, name):
    """tests/test-gemv-accuracy.cpp:184-217, tests/test-kquants-gemv.cpp:262-270."""
    f = load(os.path.join(GOLDEN, f"gemv_{name}.npz"))
    t, N, K = int(f["type"]), int(f["N"]), int(f["K"])
    y = O.gemv(t, f["w"], N, K, np.zeros(K, np.float32))
    assert np.all(y == 0.0)


def test_fp16_conversions(O):
    """tests/test-q4-0-reference.cpp:150-165 (fp16 / bf16 edge conversions)."""
    L = O.lib()
    assert L.oracle_fp16_to_f32(0x3C00) == 1.0
    assert L.oracle_fp16_to_f32(0x0001) == 2.0 ** -24
    assert L.oracle_fp16_to_f32(0x7BFF) == 65504.0
    assert L.oracle_bf16_to_f32(0x3F80) == 1.0
    assert L.oracle_bf16_to_f32(0xC000) == -2.0


def test_block_geometry(O):
    """Block sizes of include/xdna/kquants.h:180-193 (and Q4_0's 18 B / 32)."""
    want = {O.Q4_0: (32, 18), O.Q3_K: (256, 110), O.Q4_K: (256, 144), O.Q5_K: (256, 176),
            O.Q6_K: (256, 210), O.IQ3_XXS: (256, 98), O.IQ3_S: (256, 110), O.IQ2_S: (256, 82),
            O.IQ4_XS: (256, 136)}
    for t, (bv, bb) in want.items():
        assert (O.block_values(t), O.block_bytes(t)) == (bv, bb)
        assert O.row_bytes(t, 4 * bv) == 4 * bb


# ---------------------------------------------------------------- the reference, live
needs_ref = pytest.mark.skipif("not __import__('oracle').ref_available()",
                               reason="oracle/_ref not built (reference tree absent at build time)")


@needs_ref
@pytest.mark.parametrize("t", [2, 11, 12, 13, 14, 21, 23])
@pytest.mark.parametrize("shape", [(64, 1024), (48, 2048)])
def test_oracle_bit_exact_vs_reference(O, t, shape):
    from helpers import normal_weights, normal_x

    N, K = shape
    w = O.quantize(t, normal_weights(N, K, seed=11 + t))
    x = normal_x(K, seed=5)
    np.testing.assert_array_equal(O.gemv(t, w, N, K, x), O.ref_gemv(t, w, N, K, x))
    rb = O.row_bytes(t, K)
    np.testing.assert_array_equal(O.dequantize_row(t, w[rb:2 * rb], K), O.ref_dequantize_row(t, w[rb:2 * rb], K))


@needs_ref
def test_iq_tables_match_reference(O):
    grid = np.zeros(512, np.uint32)
    O.ref().ref_iq3s_grid(grid)
    kv = np.zeros(16, np.int8)
    O.ref().ref_kvalues_iq4nl(kv)
    # the reference's tables are the gguf 0.19.0 format tables the oracle's
    # generated header (oracle/gen_tables.py) was built from
    import gguf.quants as q

    q.IQ3_S.init_grid()
    g = np.ascontiguousarray(q.IQ3_S.grid.reshape(q.IQ3_S.grid_shape).astype(np.uint8))
    np.testing.assert_array_equal(g.reshape(-1).view(np.uint32), grid)
    np.testing.assert_array_equal(np.asarray(q.IQ4_NL.kvalues, dtype=np.int8).reshape(-1), kv)


@needs_ref
def test_reference_engine_matches_oracle(O):
    """The reference's own AVX2/OpenMP engine (the CPU baseline arm) agrees
    with the oracle to the reference's accuracy bar."""
    from helpers import normal_weights, normal_x

    eng = O.RefEngine()
    for t, (N, K) in [(O.Q4_0, (512, 1024)), (O.Q4_K, (512, 1024)), (O.IQ3_S, (512, 1024))]:
        w = O.quantize(t, normal_weights(N, K, seed=3))
        x = normal_x(K, seed=4)
        y = np.zeros(N, np.float32)
        eng.run(t, w, N, K, x, y)
        s = O.stats(y, O.gemv(t, w, N, K, x))
        assert s["cos"] >= 0.99999, s
    eng.close()
