#!/usr/bin/env python
"""Per-tensor decode-GEMV benchmark on the weights of a GGUF model file: the
B200 counterpart of the reference's tools/xdna-kernel-bench.cpp (which loads
one tensor of a GGUF file and times the engine on it).

Every 2-D tensor of a claimed weight type (Q4_0, Q3_K, Q4_K, Q5_K, Q6_K,
IQ2_S, IQ3_S, IQ3_XXS, IQ4_XS) is uploaded through the plugin's own path
(a B200 buffer, ggml_backend_xdna_buffer_set_tensor: pinned staging and the
GPU repack) and multiplied by a seeded N(0, 1) activation row through
ggml_backend_xdna_compute_graph.  Reported per tensor: the launch time (CUDA
events over --iters calls, one node per call), weight GB/s, and -- for
tensors up to --check-bytes -- the cosine and max-abs error against a
float64 product with the weights dequantised by the gguf package.

Usage: python xdna.cpp_b200/gguf_bench.py model.gguf [--name REGEX] [--limit N]
           [--iters 50] [--check-bytes 64000000] [--json]
"""
from __future__ import annotations

import argparse
import json
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import ggml_b200 as G  # noqa: E402


def claimed_tensors(path: str, name_re: str | None = None):
    """(name, ggml type, N, K, GGUF bytes as uint8[N * row_bytes]) of every
    2-D tensor of a claimed type, in file order."""
    from gguf import GGUFReader

    rx = re.compile(name_re) if name_re else None
    for t in GGUFReader(path).tensors:
        tid = int(t.tensor_type)
        if tid not in G.TYPE_NAME or len(t.shape) != 2 and not (len(t.shape) > 2 and all(d == 1 for d in t.shape[2:])):
            continue
        if rx and not rx.search(t.name):
            continue
        K, N = int(t.shape[0]), int(t.shape[1])  # ggml order: ne0 = K (row length), ne1 = N
        if K % G.BLOCK[tid][0]:
            continue
        raw = np.ascontiguousarray(np.asarray(t.data).reshape(-1).view(np.uint8))
        if raw.size != N * G.row_bytes(tid, K):
            continue
        yield t.name, tid, N, K, raw


def reference_product(tid: int, raw: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    import gguf
    from gguf.quants import dequantize

    qt = gguf.GGMLQuantizationType(tid)
    w = dequantize(raw.reshape(N, -1), qt).astype(np.float64).reshape(N, K)
    return (w @ x.astype(np.float64)).astype(np.float32)


def bench_tensor(torch, be, name, tid, N, K, raw, iters: int, check_bytes: int, seed: int = 7) -> dict:
    buf = G.Buffer(raw.nbytes + 2 * 4096, dev=be.dev)
    try:
        w = buf.alloc(G.tensor(tid, [K, N, 1, 1]))
        buf.set(w, raw.ctypes.data, 0, raw.nbytes)
        x = np.random.default_rng(seed).normal(0.0, 1.0, K).astype(np.float32)
        d_x = torch.from_numpy(x).cuda()
        d_y = torch.empty(N, dtype=torch.float32, device="cuda")
        xt = G.tensor(G.F32, [K, 1, 1, 1], data=d_x.data_ptr())
        node = G.mul_mat_node(w, xt, d_y.data_ptr(), N, name=name[:60])
        claimed = be.supports_op(node)
        r = {"tensor": name, "type": G.TYPE_NAME[tid], "n": N, "k": K, "weight_bytes": int(raw.nbytes),
             "claimed": bool(claimed)}
        if not claimed:
            return r
        if not be.compute([node]):
            raise RuntimeError(f"{name}: {G.last_error()}")
        stream = torch.cuda.ExternalStream(be.stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            be.compute([node])
        e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / iters
        r.update({"us_per_call": round(us, 2), "gb_s": round(raw.nbytes / (us * 1e-6) / 1e9, 1)})
        if raw.nbytes <= check_bytes:
            y = d_y.cpu().numpy().astype(np.float64)
            ref = reference_product(tid, raw, N, K, x).astype(np.float64)
            cos = float((y @ ref) / (np.linalg.norm(y) * np.linalg.norm(ref) + 1e-300))
            r.update({"cos": cos, "maxabs_rel": float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))})
        return r
    finally:
        buf.free()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("model")
    ap.add_argument("--name", help="regex on tensor names")
    ap.add_argument("--limit", type=int, default=0, help="at most this many tensors")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--check-bytes", type=int, default=64_000_000)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("-j", "--json", action="store_true")
    a = ap.parse_args()
    import torch

    if not torch.cuda.is_available():
        sys.exit("gguf_bench needs a CUDA device")
    torch.cuda.set_device(a.device)
    with G.Backend(a.device) as be:
        for i, (name, tid, N, K, raw) in enumerate(claimed_tensors(a.model, a.name)):
            if a.limit and i >= a.limit:
                break
            r = bench_tensor(torch, be, name, tid, N, K, raw, a.iters, a.check_bytes)
            if a.json:
                print(json.dumps(r), flush=True)
            else:
                chk = f"  cos {r['cos']:.9f}  maxabs/max {r['maxabs_rel']:.2e}" if "cos" in r else ""
                perf = f"{r['us_per_call']:8.2f} us {r['gb_s']:7.1f} GB/s" if "gb_s" in r else "not claimed"
                print(f"{name:40s} {r['type']:8s} {N:6d} x {K:6d}  {perf}{chk}", flush=True)


if __name__ == "__main__":
    main()
