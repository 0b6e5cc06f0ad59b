"""Generate the golden GEMV fixtures in this folder (test infrastructure).

Run in a container that has the reference tree (so ``oracle/_ref`` is built)
and the ``gguf`` package (pinned 0.19.0):

    make -C oracle all && python tests/golden/make_golden.py

For every claimed weight format it writes ``gemv_<TYPE>.npz`` holding

* ``w``    -- N x (K / block_values) seeded random blocks, in the style of the
  reference's generators (tests/test-kquants-gemv.cpp:81-217,
  tests/test-gemv-accuracy.cpp:59-86): uniform random quant bytes with
  fixed, finite fp16 scales;
* ``x``    -- K seeded N(0, 1) F32 activations;
* ``y``    -- the expected output;
* ``deq0`` -- row 0 dequantised to F32;
* ``source`` -- where ``y`` / ``deq0`` came from.

Sources:

* Q4_0: the reference's own scalar code, ``xdna::q4_0::gemv_f32`` and
  ``dequantize_row`` (src/xdna-q4-0-reference.cpp:63-97), through
  oracle/_ref/libxdna_ref.so;
* Q3_K, Q4_K, Q5_K, Q6_K, IQ4_XS, IQ3_S: the reference's ``gemv_*_ref`` and
  ``dequantize_row_*`` (include/xdna/kquants.h:290-577), same library;
* IQ3_XXS, IQ2_S: the reference has no implementation of its own (it hands
  these to ggml's CPU kernels, which are not vendored), so the third-party
  format spec stands in: ``gguf.quants.dequantize`` (gguf 0.19.0,
  gguf/quants.py:901-1056) and a float64 dot product.

The known-answer cases of the reference's tests (-264, [528, -264], 128.0,
uniform weights) need no fixture: tests/test_oracle_cpu.py builds them.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402

SHAPES = {O.Q4_0: (32, 256)}  # (N, K); the 256-value formats use (32, 512)
SEED_W, SEED_X = 20240611, 7


def random_blocks(t: int, N: int, K: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    bv, bb = O.block_values(t), O.block_bytes(t)
    nb = N * (K // bv)
    blk = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)

    def put16(col, val):
        blk[:, col] = np.asarray(val) & 0xFF
        blk[:, col + 1] = np.asarray(val) >> 8

    if t == O.Q4_0:
        put16(0, rng.choice(np.array([0x2C00, 0x3000, 0x3400, 0x3800, 0x3C00]), size=nb))
    elif t in (O.Q4_K, O.Q5_K):
        put16(0, 0x3800)
        put16(2, 0x3000)
        blk[:, 4:16] &= 0x3F
    elif t == O.Q3_K:
        put16(108, 0x3800)
    elif t == O.Q6_K:
        put16(208, 0x3800)
        blk[:, 192:208] &= 0x7F
    else:  # IQ4_XS, IQ3_S, IQ3_XXS, IQ2_S: fp16 d first
        put16(0, 0x3800)
    return blk.reshape(-1)


def gguf_expected(t: int, w: np.ndarray, N: int, K: int, x: np.ndarray):
    import gguf
    from gguf.quants import dequantize

    qt = {O.IQ3_XXS: gguf.GGMLQuantizationType.IQ3_XXS, O.IQ2_S: gguf.GGMLQuantizationType.IQ2_S}[t]
    deq = dequantize(w.reshape(N, -1), qt).astype(np.float32).reshape(N, K)
    y = (deq.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)
    return y, deq[0].copy()


def main() -> None:
    if not O.ref_available():
        sys.exit("oracle/_ref/libxdna_ref.so is not built; run `make -C oracle all` with the reference tree")
    for name, t in O.TYPES.items():
        N, K = SHAPES.get(t, (32, 512))
        w = random_blocks(t, N, K, SEED_W + t)
        x = np.random.default_rng(SEED_X + t).normal(0.0, 1.0, size=K).astype(np.float32)
        rb = O.row_bytes(t, K)
        if t in O.REF_TYPES:
            y = O.ref_gemv(t, w, N, K, x)
            deq0 = O.ref_dequantize_row(t, w[:rb], K)
            src = "reference scalar CPU code (oracle/_ref)"
        else:
            y, deq0 = gguf_expected(t, w, N, K, x)
            src = "gguf 0.19.0 dequantize + float64 dot (no in-repo reference)"
        out = os.path.join(HERE, f"gemv_{name}.npz")
        np.savez_compressed(out, w=w, x=x, y=y, deq0=deq0, N=N, K=K, type=t, source=src)
        print(f"{name:8s} N={N} K={K} -> {os.path.relpath(out, ROOT)} ({src})")


if __name__ == "__main__":
    main()
