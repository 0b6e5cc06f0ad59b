"""Shared test helpers: seeded inputs, the parity bar and GPU plumbing."""
from __future__ import annotations

import numpy as np

# Parity bar of the decode-GEMV path: cosine
# similarity >= 0.999999 and max-abs error <= 1e-4 of the output's max
# magnitude, against the reference's scalar CPU arithmetic.
COS_MIN = 0.999999
MAXABS_REL = 1e-4


def normal_weights(N: int, K: int, seed: int, sigma: float = 0.02) -> np.ndarray:
    return np.random.default_rng(seed).normal(0.0, sigma, size=(N, K)).astype(np.float32)


def normal_x(K: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).normal(0.0, 1.0, size=K).astype(np.float32)


def random_blocks(t: int, N: int, K: int, seed: int) -> np.ndarray:
    """Random valid blocks in the style of the reference's generators
    (tests/test-kquants-gemv.cpp:81-217, tests/test-gemv-accuracy.cpp:59-86):
    uniform random quant bytes with fixed, finite fp16 scales."""
    import ggml_b200 as G

    rng = np.random.default_rng(seed)
    bv, bb = G.BLOCK[t]
    nb = N * (K // bv)
    blk = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)

    def put16(col, val):
        blk[:, col] = val & 0xFF
        blk[:, col + 1] = val >> 8

    if t == G.Q4_0:
        put16(0, rng.choice(np.array([0x2C00, 0x3000, 0x3400, 0x3800, 0x3C00]), size=nb))
    elif t in (G.Q4_K, G.Q5_K):
        put16(0, 0x3800)  # d = 0.5
        put16(2, 0x3000)  # dmin = 0.125
        blk[:, 4:16] &= 0x3F
    elif t == G.Q3_K:
        put16(108, 0x3800)
    elif t == G.Q6_K:
        put16(208, 0x3800)
        blk[:, 192:208] &= 0x7F
    elif t in (G.IQ4_XS, G.IQ3_S, G.IQ3_XXS, G.IQ2_S):
        put16(0, 0x3800)
    return blk.reshape(-1)


def check_parity(y: np.ndarray, y_ref: np.ndarray, what: str = "") -> dict:
    import oracle as O

    s = O.stats(y, y_ref)
    assert s["cos"] >= COS_MIN, f"{what}: cos {s['cos']:.9f} < {COS_MIN} ({s})"
    assert s["maxabs_rel"] <= MAXABS_REL, f"{what}: maxabs/max|y| {s['maxabs_rel']:.3e} > {MAXABS_REL} ({s})"
    return s


def to_dev(torch, a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gemv_gpu(torch, G, t: int, raw: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    """GGUF bytes -> device -> b200_repack -> b200_gemv, on torch's current stream."""
    stream = torch.cuda.current_stream().cuda_stream
    d_raw = to_dev(torch, raw)
    d_pk = torch.empty_like(d_raw)
    d_x = to_dev(torch, x)
    d_y = torch.full((max(N, 1),), float("nan"), dtype=torch.float32, device="cuda")
    G.check(G.lib().b200_repack(t, d_raw.data_ptr(), d_pk.data_ptr(), N, K, stream), "repack")
    G.check(G.lib().b200_gemv(t, d_pk.data_ptr(), d_x.data_ptr(), d_y.data_ptr(), N, K, stream, 0), "gemv")
    torch.cuda.synchronize()
    return d_y[:N].cpu().numpy()
