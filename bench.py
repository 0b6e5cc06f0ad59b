#!/usr/bin/env python
"""Decode-GEMV benchmark of the B200 backend (driver contract: one JSON line).

Headline workload (the one the metric quotes at
1/2/4/8 B200): a random-init Llama-3-70B-shaped Q4_K layer stack, batch 1.
One step = one decode token = the 561 single-row MUL_MATs the backend claims
(80 layers x q, k, v, o, gate, up, down + lm_head), 39,094,714,368 weight
bytes, chained through device activations (q/k/v read h, o reads q, gate/up
read o, down reads gate and writes h, lm_head reads h).  Non-MUL_MAT ops
(norms, RoPE, attention, SwiGLU) stay with the host framework in this plugin
model and are not part of the step.  With N GPUs every weight is row-sharded
(rank r owns rows [r N/W, (r+1) N/W)) and each launch is completed inside
ggml_backend_xdna_compute_graph: the GEMV stores its rows into the peers'
exchange buffers over NVLink and a gather kernel assembles the full outputs
(an NCCL all-gather of the F32 slices where the exchange is unavailable).

  value : aggregate weight GB/s of the step with activations resident in HBM
          (CUDA events on the backend stream, max over ranks)
  e2e   : the same through the public C ABI with the token's input vector
          copied from pinned host memory and the logits read back every step
  --impl reference : the reference's own CPU GEMV engine (oracle/_ref,
          XdnaGemvEngine::run_quant, AVX2 + OpenMP) on a bounded sample of the
          same workload (one layer's seven matmuls), rank 0 only

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
import zlib

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "xdna.cpp_b200"))

METRIC = "GEMV HBM GB/s (% of 8 TB/s) per quant type; decode tok/s at 1/2/4/8 B200"
Q4_K = 12
HIDDEN, KV, FF, VOCAB, LAYERS = 8192, 1024, 28672, 128256, 80
LAYER_MATS = [("q", HIDDEN, HIDDEN), ("k", KV, HIDDEN), ("v", KV, HIDDEN), ("o", HIDDEN, HIDDEN),
              ("gate", FF, HIDDEN), ("up", FF, HIDDEN), ("down", HIDDEN, FF)]
NOMINAL_HBM_GBS = 8000.0


def row_bytes_q4k(K: int) -> int:
    return (K // 256) * 144


WEIGHT_BYTES_PER_TOKEN = (LAYERS * sum(N * row_bytes_q4k(K) for _, N, K in LAYER_MATS)
                          + VOCAB * row_bytes_q4k(HIDDEN))
MATMULS_PER_TOKEN = LAYERS * len(LAYER_MATS) + 1
LAUNCHES_PER_TOKEN = LAYERS * 4 + 1  # q/k/v fused, o, gate/up fused, down; lm_head


# ------------------------------------------------------------------ plumbing
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            torch.cuda.set_device(self.local_rank)
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local_rank))
            self.pg = dist

    def broadcast_bytes(self, b: bytes | None) -> bytes:
        if self.world == 1:
            return b
        import torch

        t = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if self.rank == 0:
            t.copy_(torch.frombuffer(bytearray(b), dtype=torch.uint8))
        self.pg.broadcast(t, 0)
        return bytes(t.cpu().numpy().tobytes())

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def barrier(self) -> None:
        if self.world > 1:
            self.pg.barrier()

    def close(self) -> None:
        if self.pg is not None:
            self.pg.destroy_process_group()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9 and f[1].replace(".", "").isdigit():
                    rows.append(f)
        except OSError:
            pass
        finally:
            if self.path and os.path.exists(self.path):
                os.remove(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def profiled_traffic() -> tuple[int | None, str]:
    """DRAM bytes (read + write) of one step's GEMV launches, from the committed
    ncu launch-list summary of this workload (profiles/decode70b_q4k_launches.md)."""
    p = os.path.join(ROOT, "profiles", "decode70b_q4k_launches.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_step:"):
                return int(line.split(":")[1].split()[0]), "profiles/decode70b_q4k_launches.md"
    except (OSError, ValueError):
        pass
    return None, "no profile"


def measured_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        v = float(json.load(open(p))["hbm_gbs"])
        return v, "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ------------------------------------------------------------- CPU baseline
def reference_cpu_sample(seconds: float, seed: int = 1) -> dict:
    """The reference's CPU engine on one Llama-3-70B-shaped Q4_K layer (its
    seven matmuls, 481 MB of weights), repeated for about `seconds`."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    kind = "reference" if O.ref_available() else "port"
    rng = np.random.default_rng(seed)
    mats = []
    for name, N, K in LAYER_MATS:
        W = rng.normal(0.0, 0.02, size=(N, K)).astype(np.float32)
        q = O.quantize(O.Q4_K, W, nthreads=os.cpu_count() or 8)
        del W
        mats.append((name, N, K, q, rng.normal(0.0, 1.0, K).astype(np.float32), np.empty(N, np.float32)))
    layer_bytes = sum(q.nbytes for _, _, _, q, _, _ in mats)
    if kind == "reference":
        eng = O.RefEngine()

        def run_layer():
            for _, N, K, q, x, y in mats:
                eng.run(O.Q4_K, q, N, K, x, y)
        threads = min(8, os.cpu_count() or 8)  # run_quant's AVX2 path uses num_threads(8)
    else:
        threads = os.cpu_count() or 8

        def run_layer():
            for _, N, K, q, x, y in mats:
                y[:] = O.gemv(O.Q4_K, q, N, K, x, nthreads=threads)
    run_layer()  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        run_layer()
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = n * layer_bytes / el / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind,
            "tok_s": gbs * 1e9 / WEIGHT_BYTES_PER_TOKEN,
            "sample": f"{n} x one 70B-shaped Q4_K layer (q,k,v,o,gate,up,down: {layer_bytes} weight bytes) "
                      f"on {threads} host threads, {el:.1f} s; tok/s extrapolated to 561 matmuls "
                      f"({WEIGHT_BYTES_PER_TOKEN} B)",
            "seconds": el}


def run_reference_arm(args, dist: Dist) -> None:
    if dist.rank != 0:
        return
    # each step is one layer sample; keep the whole run to a few minutes
    per_step = max(0.5, min(5.0, 60.0 / max(1, args.steps + args.warmup)))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    base = reference_cpu_sample(per_step * max(1, args.steps))
    line = {"metric": METRIC, "impl": "reference", "value": base["value"], "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * base["seconds"] / max(1, args.steps),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic N(0,0.02) weights quantised to Q4_K, N(0,1) activations",
            "config": {"workload": "llama3-70b-shaped Q4_K decode matmuls (one-layer CPU sample)",
                       "tok_s": base["tok_s"]},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ B200 arm
class Model:
    """Per-rank shards of the 70B-shaped Q4_K stack in one B200 buffer, plus
    the device activations and the 561-node compute graph."""

    def __init__(self, G, torch, be, world: int, rank: int, distinct_layers: int = 2):
        self.G, self.torch, self.be = G, torch, be
        self.world, self.rank = world, rank
        specs = []  # (layer, name, N_full, K)
        for layer in range(LAYERS):
            for name, N, K in LAYER_MATS:
                specs.append((layer, name, N, K))
        specs.append((LAYERS, "lm_head", VOCAB, HIDDEN))
        self.local_bytes = 0
        for _, _, N, K in specs:
            _, nr = G.shard_rows(N, world, rank)
            self.local_bytes += nr * row_bytes_q4k(K)
        align = 4096
        self.buf = G.Buffer(self.local_bytes + align * (len(specs) + 2), dev=torch.cuda.current_device())
        self.weights = {}
        src_of = {}
        for layer, name, N, K in specs:
            _, nr = G.shard_rows(N, world, rank)
            t = self.buf.alloc(G.tensor(Q4_K, [K, nr, 1, 1], name=f"{name}.{layer}"))
            self.weights[(layer, name)] = t
            key = (name, layer % distinct_layers if layer < LAYERS else -1)
            if key not in src_of:
                src_of[key] = (layer, name)
                self._generate(t, nr, K, seed=zlib.crc32(f"{key[0]}:{key[1]}:{rank}".encode()))
            else:
                G.Buffer.copy(self.weights[src_of[key]], t)
        dev = "cuda"
        f32 = torch.float32
        self.act = {"h": torch.zeros(HIDDEN, dtype=f32, device=dev), "q": torch.zeros(HIDDEN, dtype=f32, device=dev),
                    "k": torch.zeros(KV, dtype=f32, device=dev), "v": torch.zeros(KV, dtype=f32, device=dev),
                    "o": torch.zeros(HIDDEN, dtype=f32, device=dev), "gate": torch.zeros(FF, dtype=f32, device=dev),
                    "up": torch.zeros(FF, dtype=f32, device=dev), "logits": torch.zeros(VOCAB, dtype=f32, device=dev)}
        self.act["h"].normal_()
        self._keep = []
        self.nodes = self._build_nodes(self.act["h"].data_ptr(), self.act["logits"].data_ptr())
        # e2e graph: token input from pinned host memory, logits back to pinned host memory
        self.h_host = torch.empty(HIDDEN, dtype=f32, pin_memory=True)
        self.h_host.normal_()
        self.logits_host = torch.empty(VOCAB, dtype=f32, pin_memory=True)
        self.nodes_e2e = self._build_nodes(self.h_host.data_ptr(), self.logits_host.data_ptr(), first_x_host=True)

    def _generate(self, t, nr: int, K: int, seed: int) -> None:
        torch, G = self.torch, self.G
        w = torch.empty(nr * K, dtype=torch.float32, device="cuda")
        G.check(G.lib().b200_fill_normal(w.data_ptr(), w.numel(), seed, 0.02, 0), "fill_normal")
        q = torch.empty(nr * row_bytes_q4k(K), dtype=torch.uint8, device="cuda")
        G.check(G.lib().b200_quantize(Q4_K, w.data_ptr(), q.data_ptr(), nr, K, 0), "quantize")
        torch.cuda.synchronize()
        del w
        self.buf.set_device(t, q.data_ptr(), 0, q.numel())

    def _act_tensor(self, name_or_ptr, n: int):
        G = self.G
        ptr = name_or_ptr if isinstance(name_or_ptr, int) else self.act[name_or_ptr].data_ptr()
        t = G.tensor(G.F32, [n, 1, 1, 1], data=ptr)
        self._keep.append(t)
        return t

    def _node(self, layer, name, x, y_ptr, n_full):
        G = self.G
        w = self.weights[(layer, name)]
        node = G.mul_mat_node(w, x, y_ptr, n_full, name=f"{name}.{layer}")
        self._keep.append(node)
        return node

    def _build_nodes(self, h0_ptr: int, logits_ptr: int, first_x_host: bool = False):
        a = self.act
        nodes = []
        h_in = self._act_tensor(h0_ptr, HIDDEN)
        h = self._act_tensor("h", HIDDEN)
        for layer in range(LAYERS):
            x = h_in if layer == 0 else h
            nodes.append(self._node(layer, "q", x, a["q"].data_ptr(), HIDDEN))
            nodes.append(self._node(layer, "k", x, a["k"].data_ptr(), KV))
            nodes.append(self._node(layer, "v", x, a["v"].data_ptr(), KV))
            nodes.append(self._node(layer, "o", self._act_tensor("q", HIDDEN), a["o"].data_ptr(), HIDDEN))
            xo = self._act_tensor("o", HIDDEN)
            nodes.append(self._node(layer, "gate", xo, a["gate"].data_ptr(), FF))
            nodes.append(self._node(layer, "up", xo, a["up"].data_ptr(), FF))
            nodes.append(self._node(layer, "down", self._act_tensor("gate", FF), a["h"].data_ptr(), HIDDEN))
        nodes.append(self._node(LAYERS, "lm_head", h, logits_ptr, VOCAB))
        return nodes


def time_steps(torch, be, nodes, steps: int) -> float:
    """Device time (ms) of `steps` compute_graph calls, CUDA events on the backend stream."""
    s = torch.cuda.ExternalStream(be.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    be.synchronize()
    torch.cuda.nvtx.range_push("timed")  # lets a profiler select the timed launches
    e0.record(s)
    for _ in range(steps):
        if not be.compute(nodes):
            raise RuntimeError(f"compute_graph failed: {be_last_error()}")
    e1.record(s)
    torch.cuda.nvtx.range_pop()
    e1.synchronize()
    return e0.elapsed_time(e1)


def be_last_error() -> str:
    import ggml_b200 as G

    return G.last_error()


def kernel_only_ms(torch, G, model, steps: int) -> float:
    """Device time of one step's GEMV launches alone (no exchange, no host
    work), for the roofline of the dominant kernel when the step itself also
    holds the row exchange (N > 1): the launches compute_graph makes -- q/k/v
    and gate/up fused (b200_gemv_multi), o, down and lm_head single
    (b200_gemv), each with its x preparation -- captured once as a CUDA graph
    and replayed."""
    import ctypes as C

    a = model.act
    plan = []  # (weights, outputs, rows, x, K) per launch
    groups = [(("q", "k", "v"), "h"), (("o",), "q"), (("gate", "up"), "o"), (("down",), "gate")]
    for layer in range(LAYERS):
        for names, x in groups:
            ws = [model.weights[(layer, n)] for n in names]
            ys = [a[{"down": "h"}.get(n, n)].data_ptr() for n in names]
            plan.append(([w.data for w in ws], ys, [w.ne[1] for w in ws], a[x].data_ptr(), ws[0].ne[0]))
    w = model.weights[(LAYERS, "lm_head")]
    plan.append(([w.data], [a["logits"].data_ptr()], [w.ne[1]], a["h"].data_ptr(), HIDDEN))
    L = G.lib()
    packed = []
    for wps, yps, ns, xp, k in plan:
        n = len(wps)
        packed.append((n, (C.c_void_p * n)(*wps), (C.c_void_p * n)(*yps), (C.c_int64 * n)(*ns), xp, k))

    def step(stream_handle: int):
        for n, wps, yps, ns, xp, k in packed:
            if n == 1:
                rc = L.b200_gemv(Q4_K, wps[0], xp, yps[0], ns[0], k, stream_handle, 1)
            else:
                rc = L.b200_gemv_multi(Q4_K, wps, yps, ns, n, xp, k, stream_handle, 1)
            if rc:
                raise RuntimeError(G.last_error())

    # one step captured as a CUDA graph, so host launch cost does not enter the measurement
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        step(side.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step(side.cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    e0.record(cur)
    for _ in range(steps):
        graph.replay()
    e1.record(cur)
    e1.synchronize()
    del graph
    return e0.elapsed_time(e1) / steps


def run_b200_arm(args, dist: Dist) -> None:
    import torch

    import ggml_b200 as G

    G.lib()
    torch.cuda.set_device(dist.local_rank)
    t_setup = time.perf_counter()
    nccl_id = dist.broadcast_bytes(G.nccl_unique_id() if dist.rank == 0 else None) if dist.world > 1 else None
    be = G.Backend(dist.local_rank, dist.world, dist.rank, nccl_id)
    model = Model(G, torch, be, dist.world, dist.rank)
    torch.cuda.synchronize()
    setup_s = time.perf_counter() - t_setup
    dist.barrier()

    for _ in range(args.warmup):
        if not be.compute(model.nodes):
            raise RuntimeError(f"compute_graph failed: {G.last_error()}")
    be.synchronize()
    dist.barrier()
    with ClockSampler(dist.local_rank) as clk:
        ms = time_steps(torch, be, model.nodes, args.steps)
    dist.barrier()
    ms_step = dist.max(ms / args.steps)

    # end to end through the C ABI with host input / output every step
    for _ in range(max(1, args.warmup // 2)):
        be.compute(model.nodes_e2e)
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        if not be.compute(model.nodes_e2e):
            raise RuntimeError(f"compute_graph (e2e) failed: {G.last_error()}")
    e2e_ms = dist.max((time.perf_counter() - t0) * 1000.0 / args.steps)
    dist.barrier()

    # the dominant kernel's device time per step.  On one GPU the timed step is
    # the GEMV chain alone (each launch prepares the next one's x; one x
    # preparation kernel per step), so its own CUDA-event time is used.  With
    # N GPUs the step also holds the row exchange: the GEMV launches are timed
    # alone instead (b200_gemv / b200_gemv_multi, an x preparation per launch).
    if dist.world == 1:
        k_ms, k_src = ms_step, "the timed compute_graph step (CUDA events on the backend stream)"
    else:
        k_ms = dist.max(kernel_only_ms(torch, G, model, max(2, args.steps // 2)))
        k_src = "GEMV launches alone per step (b200_gemv / b200_gemv_multi replayed as a CUDA graph)"
    peak, peak_src = measured_peak()
    traffic, traffic_src = profiled_traffic() if dist.world == 1 else (None, "profiled at N=1 only")
    achieved = model.local_bytes / (k_ms * 1e-3) / 1e9

    cpu = None
    if dist.rank == 0 and dist.world == 1:
        cpu = reference_cpu_sample(seconds=args.cpu_seconds)
    dist.barrier()

    if dist.rank == 0:
        value = WEIGHT_BYTES_PER_TOKEN / (ms_step * 1e-3) / 1e9
        e2e_gbs = WEIGHT_BYTES_PER_TOKEN / (e2e_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: random-init N(0,0.02) weights quantised on the GPU to Q4_K, N(0,1) activations",
            "config": {
                "workload": "llama3-70b-shaped Q4_K decode: 561 M=1 MUL_MATs per token "
                            "(80 layers x q,k,v,o,gate,up,down + lm_head), rows sharded over N GPUs, outputs exchanged "
                            "over NVLink by the GEMV and a gather kernel (NCCL all-gather fallback)",
                "weight_bytes_per_token": WEIGHT_BYTES_PER_TOKEN, "matmuls_per_token": MATMULS_PER_TOKEN,
                "batch": 1, "parallelism": f"rows{dist.world}",
                "tok_s": round(1000.0 / ms_step, 3),
                "pct_of_8tbs": round(100.0 * value / (NOMINAL_HBM_GBS * dist.world), 2),
                "l2": "per-step weights (39 GB) exceed the 126 MB L2; no flush needed",
                "setup_s": round(setup_s, 1),
            },
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "tok_s": round(1000.0 / e2e_ms, 3),
                    "h2d_bytes_per_step": 3 * HIDDEN * 4, "d2h_bytes_per_step": VOCAB * 4,
                    "path": "ggml_backend_xdna_compute_graph, token input from pinned host memory, logits to host"},
            "roofline": {"bound": "hbm", "kernel": "gemv_mma_kernel<12> (Q4_K)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": traffic, "traffic_unit": "bytes per step (all GEMV launches)",
                         "traffic_source": traffic_src, "algorithmic_bytes_per_step": model.local_bytes,
                         "per_launch_note": f"{LAUNCHES_PER_TOKEN} GEMV launches per step (q/k/v and gate/up "
                         "fused); achieved = local weight bytes per step / device time per step of " + k_src},
            "clocks": clk.summary(),
            # one GPU: 321 gemv_mma_kernel launches + one xprep_kernel per step
            # (every later launch's x is prepared by the launch before it);
            # N GPUs: also one xchg_gather_kernel per launch (it prepares the
            # next launch's x); NCCL's kernels, on the fallback path, not counted
            "gpu_launches": args.steps * (LAUNCHES_PER_TOKEN * (1 if dist.world == 1 else 2) + 1),
        }
        if cpu is not None:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    be.close()
    model.buf.free()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    dist = Dist()
    try:
        if args.impl == "reference":
            run_reference_arm(args, dist)
        else:
            run_b200_arm(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
