#!/usr/bin/env python
"""Per-format decode-GEMV bandwidth benchmark: the B200 counterpart of the
reference's ``xdna-bandwidth-bench -m gemv`` (tools/xdna-bandwidth-bench.cpp:
706-828).  It reports GB/s of weight bytes per launch, as the reference does,
plus the fraction of the nominal 8 TB/s and of the measured HBM copy peak.

Timing differs from the reference's wall-clock loop in two ways that make
the number an HBM number rather than a cache number: launches are timed with
CUDA events on the launching stream, and the kernel rotates through enough
device copies of the weights to exceed twice the 126 MB L2, so every launch
streams its weights from HBM.

Weights: Q4_0 and Q4_K are drawn N(0, 0.02) and quantised on the GPU
(b200_fill_normal + b200_quantize); the other formats use seeded uniform
random quant bytes with fixed, finite fp16 scales (timing does not depend
on the values).  x ~ N(0, 1).

Usage: python xdna.cpp_b200/gemv_bench.py [-t Q4_K] [-n 28672] [-k 8192]
           [--iters 100] [-w 5] [--graph] [--json]
       python xdna.cpp_b200/gemv_bench.py --sweep     (every claimed format
           at the configs' shapes)
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import ggml_b200 as G  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
NOMINAL_GBS = 8000.0

# Q4_0 at 4096^2, 8192^2, 17408x5120; every other format at
# 11008x2048 and 2048x11008 (N x K), K rounded down to the 256-value block
SWEEP = ([("Q4_0", 4096, 4096), ("Q4_0", 8192, 8192), ("Q4_0", 17408, 5120)]
         + [(name, n, k) for name in ("Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ2_S", "IQ3_S", "IQ3_XXS", "IQ4_XS")
            for n, k in ((11008, 2048), (2048, 11008 // 256 * 256))]
         + [("Q4_K", 28672, 8192), ("Q4_K", 8192, 28672), ("Q4_K", 128256, 8192)])


def measured_peak() -> float | None:
    try:
        return float(json.load(open(os.path.join(HERE, "..", "MEASURED_PEAKS.json")))["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def random_blocks(t: int, n: int, k: int, seed: int) -> np.ndarray:
    bv, bb = G.BLOCK[t]
    nb = n * (k // bv)
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    d_off = {G.Q3_K: 108, G.Q6_K: 208}.get(t, 0)  # fp16 d: first field, or last for Q3_K / Q6_K
    blk[:, d_off], blk[:, d_off + 1] = 0x00, 0x38  # d = 0.5
    if t in (G.Q4_K, G.Q5_K):
        blk[:, 2], blk[:, 3] = 0x00, 0x30          # dmin = 0.125
    return blk.reshape(-1)


def make_weights(torch, t: int, n: int, k: int, stream: int, seed: int):
    """One packed (kernel-layout) copy of an n x k weight matrix on the device."""
    L = G.lib()
    nbytes = n * G.row_bytes(t, k)
    raw = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    if t in (G.Q4_0, G.Q4_K):
        f = torch.empty(n * k, dtype=torch.float32, device="cuda")
        G.check(L.b200_fill_normal(f.data_ptr(), n * k, seed, 0.02, stream), "fill_normal")
        G.check(L.b200_quantize(t, f.data_ptr(), raw.data_ptr(), n, k, stream), "quantize")
        del f
    else:
        raw.copy_(torch.from_numpy(random_blocks(t, n, k, seed)))
    packed = torch.empty_like(raw)
    G.check(L.b200_repack(t, raw.data_ptr(), packed.data_ptr(), n, k, stream), "repack")
    torch.cuda.synchronize()
    return packed


def bench_one(torch, name: str, n: int, k: int, iters: int, warmup: int, graph: bool, seed: int = 42) -> dict:
    t = G.CLAIMED[name]
    L = G.lib()
    s = torch.cuda.Stream()
    sh = s.cuda_stream
    nbytes = n * G.row_bytes(t, k)
    copies = max(1, -(-2 * L2_BYTES // nbytes))  # rotate past 2x L2
    with torch.cuda.stream(s):
        ws = [make_weights(torch, t, n, k, sh, seed + i) for i in range(min(copies, 1))]
        while len(ws) < copies:
            ws.append(ws[0].clone())  # same bytes, distinct addresses
        x = torch.randn(k, dtype=torch.float32, device="cuda", generator=torch.Generator("cuda").manual_seed(seed))
        y = torch.empty(n, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def launch(i: int) -> None:
        rc = L.b200_gemv(t, ws[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), n, k, sh, 1)
        if rc:
            raise RuntimeError(G.last_error())

    for i in range(max(3, warmup)):
        launch(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(iters):
                launch(i)
        with torch.cuda.stream(s):
            g.replay()
            torch.cuda.synchronize()
            e0.record(s)
            g.replay()
            e1.record(s)
    else:
        e0.record(s)
        for i in range(iters):
            launch(i)
        e1.record(s)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / iters
    gbs = nbytes / (us * 1e-6) / 1e9
    peak = measured_peak()
    return {"type": name, "n": n, "k": k, "weight_bytes": nbytes, "us_per_launch": round(us, 2),
            "gb_s": round(gbs, 1), "pct_of_8tbs": round(100.0 * gbs / NOMINAL_GBS, 1),
            "frac_of_measured": round(gbs / peak, 4) if peak else None, "copies": copies,
            "launch": "cuda graph" if graph else "stream", "iters": iters}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("-t", "--type", default="Q4_K", choices=sorted(G.CLAIMED))
    ap.add_argument("-n", "--dim-n", type=int, default=28672)
    ap.add_argument("-k", "--dim-k", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("-w", "--warmup", type=int, default=5)
    ap.add_argument("--graph", action="store_true", help="launch the timed loop as one CUDA graph")
    ap.add_argument("--sweep", action="store_true", help="every format at the configs' shapes")
    ap.add_argument("-j", "--json", action="store_true", help="one JSON object per line")
    a = ap.parse_args()
    import torch

    if not torch.cuda.is_available():
        sys.exit("gemv_bench needs a CUDA device")
    cases = SWEEP if a.sweep else [(a.type, a.dim_n, a.dim_k)]
    for name, n, k in cases:
        r = bench_one(torch, name, n, k, a.iters, a.warmup, a.graph)
        if a.json:
            print(json.dumps(r), flush=True)
        else:
            print(f"{name:8s} {n:6d} x {k:6d}  {r['us_per_launch']:8.2f} us  {r['gb_s']:7.1f} GB/s  "
                  f"{r['pct_of_8tbs']:5.1f}% of 8 TB/s  frac(measured) {r['frac_of_measured']}", flush=True)


if __name__ == "__main__":
    main()
