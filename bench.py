#!/usr/bin/env python
"""Decode-GEMV benchmark of the B200 backend (driver contract: one JSON line).

Headline workload (the one the metric quotes at
1/2/4/8 B200): a random-init Llama-3-70B-shaped Q4_K layer stack, batch 1.
One step = one decode token = the 561 single-row MUL_MATs the backend claims
(80 layers x q, k, v, o, gate, up, down + lm_head), 39,094,714,368 weight
bytes, chained through device activations (q/k/v read h_l, o reads q_l,
gate/up read o_l, down reads gate_l and writes h_{l+1}, lm_head reads h_80;
every layer has its own activation vectors, so after a step every node's
input and output can be read back and checked).  Non-MUL_MAT ops (norms,
RoPE, attention, SwiGLU) stay with the host framework in this plugin model
and are not part of the step.  With N GPUs every weight is row-sharded
(rank r owns rows [r N/W, (r+1) N/W)) and each launch is completed inside
ggml_backend_xdna_compute_graph: the GEMV stores its rows into the peers'
exchange buffers over NVLink and a gather kernel assembles the full outputs
(an NCCL all-gather of the F32 slices where the exchange is unavailable).

  value : aggregate weight GB/s of the step with activations resident in HBM
          (CUDA events on the backend stream, max over ranks)
  e2e   : the same through the public C ABI with the token's input vector
          copied from pinned host memory and the logits read back every step
  check : after timing, the outputs of one more step of the timed node list
          (layers 0 and 1) and an lm_head call on layer 1's output, against
          the CPU oracle on their actual inputs; a miss fails the run
  config.per_format : (N = 1) every claimed format at the configs[0-2]
          shapes: GB/s, fraction of the measured HBM peak, cos / max-abs
          against the oracle, and the reference's CPU engine beside it
  config.qwen3b_decode : (N = 1) configs[3], greedy decode of the
          Qwen2.5-3B-shaped Q4_0 model through the plugin with host ops: tok/s
          and the 32-token greedy match against the oracle-driven decode
  --impl reference : the reference's own CPU GEMV engine (oracle/_ref,
          XdnaGemvEngine::run_quant, AVX2 + OpenMP) on a bounded sample of the
          same workload (one layer's seven matmuls), rank 0 only

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                       [--layers L] [--profile-run]
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
L2_BYTES = 126 * 1024 * 1024
# the north_star parity bar per GEMV
COS_MIN, MAXABS_REL = 0.999999, 1e-4


def row_bytes_q4k(K: int) -> int:
    return (K // 256) * 144


def weight_bytes_per_token(layers: int) -> int:
    return layers * sum(N * row_bytes_q4k(K) for _, N, K in LAYER_MATS) + VOCAB * row_bytes_q4k(HIDDEN)


def launches_per_token(layers: int) -> int:
    return layers * 4 + 1  # q/k/v fused, o, gate/up fused, down; lm_head


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

    def reduce(self, v: float, op: str) -> float:
        if self.world == 1:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX if op == "max" else self.pg.ReduceOp.MIN)
        return float(t.item())

    def max(self, v: float) -> float:
        return self.reduce(v, "max")

    def barrier(self) -> None:
        if self.world > 1:
            self.pg.barrier()

    def close(self) -> None:
        if self.pg is not None:
            self.pg.destroy_process_group()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

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


def profiled_traffic_ratio() -> tuple[float | None, str]:
    """DRAM bytes (read + write) per algorithmic weight byte of the GEMV
    launches, from the committed single-kernel ncu capture of a two-layer
    model of this workload (profiles/gemv_mma_q4k_decode_traffic.md)."""
    name = "profiles/gemv_mma_q4k_decode_traffic.md"
    try:
        for line in open(os.path.join(ROOT, name)):
            if line.startswith("traffic_ratio:"):
                return float(line.split(":")[1].split()[0]), name
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


def oracle_module():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    return O


def parity(O, y: np.ndarray, ref: np.ndarray) -> dict:
    s = O.stats(y, ref)
    return {"cos": round(s["cos"], 9), "maxabs_rel": float(f"{s['maxabs_rel']:.3e}"),
            "ok": bool(s["cos"] >= COS_MIN and s["maxabs_rel"] <= MAXABS_REL)}


# ------------------------------------------------------------- CPU baseline
def reference_cpu_sample(seconds: float, seed: int = 1) -> dict:
    """The reference's CPU engine on one Llama-3-70B-shaped Q4_K layer (its
    seven matmuls, 481 MB of weights), repeated for about `seconds`."""
    O = oracle_module()
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
    wbt = weight_bytes_per_token(LAYERS)
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind, "tok_s": gbs * 1e9 / wbt,
            "sample": f"{n} x one 70B-shaped Q4_K layer (q,k,v,o,gate,up,down: {layer_bytes} weight bytes) "
                      f"on {threads} host threads, {el:.1f} s; tok/s extrapolated to 561 matmuls ({wbt} B)",
            "seconds": el}


def run_reference_arm(args, dist: Dist) -> None:
    if dist.rank != 0:
        return
    # each step is one layer sample; keep the whole run to a few minutes
    per_step = max(0.5, min(5.0, 60.0 / max(1, args.steps + args.warmup)))
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
    """Per-rank shards of the 70B-shaped Q4_K stack in one B200 buffer, the
    per-layer device activations and the step's node list."""

    def __init__(self, G, torch, be, world: int, rank: int, layers: int = LAYERS, distinct_layers: int = 2):
        self.G, self.torch, self.be = G, torch, be
        self.world, self.rank, self.layers = world, rank, layers
        self.distinct = distinct_layers
        specs = []  # (layer, name, N_full, K)
        for layer in range(layers):
            for name, N, K in LAYER_MATS:
                specs.append((layer, name, N, K))
        specs.append((layers, "lm_head", VOCAB, HIDDEN))
        self.specs = specs
        self.local_bytes = 0
        for _, _, N, K in specs:
            _, nr = G.shard_rows(N, world, rank)
            self.local_bytes += nr * row_bytes_q4k(K)
        align = 4096
        self.buf = G.Buffer(self.local_bytes + align * (len(specs) + 2), dev=torch.cuda.current_device())
        self.weights = {}
        self.src_of = {}
        for layer, name, N, K in specs:
            _, nr = G.shard_rows(N, world, rank)
            t = self.buf.alloc(G.tensor(Q4_K, [K, nr, 1, 1], name=f"{name}.{layer}"))
            self.weights[(layer, name)] = t
            key = self.weight_key(layer, name)
            if key not in self.src_of:
                self.src_of[key] = (layer, name)
                self._generate(t, nr, K, seed=zlib.crc32(f"{key[0]}:{key[1]}:{rank}".encode()))
            else:
                G.Buffer.copy(self.weights[self.src_of[key]], t)
        f32 = torch.float32
        z = lambda n: torch.zeros(n, dtype=f32, device="cuda")  # noqa: E731
        # h[l] is layer l's input (h[layers] feeds lm_head); every layer has its own q..up
        self.h = [z(HIDDEN) for _ in range(layers + 1)]
        self.acts = [{"q": z(HIDDEN), "k": z(KV), "v": z(KV), "o": z(HIDDEN), "gate": z(FF), "up": z(FF)}
                     for _ in range(layers)]
        self.logits = z(VOCAB)
        self.h[0].normal_()
        self._keep = []
        self.nodes = self._build_nodes(self.h[0].data_ptr(), self.logits.data_ptr())
        # e2e list: token input from pinned host memory, logits back to pinned host memory
        self.h_host = torch.empty(HIDDEN, dtype=f32, pin_memory=True)
        self.h_host.normal_()
        self.logits_host = torch.empty(VOCAB, dtype=f32, pin_memory=True)
        self.nodes_e2e = self._build_nodes(self.h_host.data_ptr(), self.logits_host.data_ptr())

    def weight_key(self, layer: int, name: str):
        return (name, layer % self.distinct if layer < self.layers else -1)

    def _generate(self, t, nr: int, K: int, seed: int) -> None:
        torch, G = self.torch, self.G
        w = torch.empty(nr * K, dtype=torch.float32, device="cuda")
        G.check(G.lib().b200_fill_normal(w.data_ptr(), w.numel(), seed, 0.02, 0), "fill_normal")
        q = torch.empty(nr * row_bytes_q4k(K), dtype=torch.uint8, device="cuda")
        G.check(G.lib().b200_quantize(Q4_K, w.data_ptr(), q.data_ptr(), nr, K, 0), "quantize")
        torch.cuda.synchronize()
        del w
        self.buf.set_device(t, q.data_ptr(), 0, q.numel())

    def _vec(self, ptr: int, n: int):
        t = self.G.tensor(self.G.F32, [n, 1, 1, 1], data=ptr)
        self._keep.append(t)
        return t

    def _node(self, layer, name, x, y_ptr, n_full):
        node = self.G.mul_mat_node(self.weights[(layer, name)], x, y_ptr, n_full, name=f"{name}.{layer}")
        self._keep.append(node)
        return node

    def _build_nodes(self, h0_ptr: int, logits_ptr: int):
        nodes = []
        for layer in range(self.layers):
            a = self.acts[layer]
            x = self._vec(h0_ptr if layer == 0 else self.h[layer].data_ptr(), HIDDEN)
            for name, n in (("q", HIDDEN), ("k", KV), ("v", KV)):
                nodes.append(self._node(layer, name, x, a[name].data_ptr(), n))
            nodes.append(self._node(layer, "o", self._vec(a["q"].data_ptr(), HIDDEN), a["o"].data_ptr(), HIDDEN))
            xo = self._vec(a["o"].data_ptr(), HIDDEN)
            nodes.append(self._node(layer, "gate", xo, a["gate"].data_ptr(), FF))
            nodes.append(self._node(layer, "up", xo, a["up"].data_ptr(), FF))
            nodes.append(self._node(layer, "down", self._vec(a["gate"].data_ptr(), FF), self.h[layer + 1].data_ptr(),
                                    HIDDEN))
        nodes.append(self._node(self.layers, "lm_head", self._vec(self.h[self.layers].data_ptr(), HIDDEN),
                                logits_ptr, VOCAB))
        return nodes

    def raw_weights(self, layer: int, name: str) -> np.ndarray:
        """GGUF bytes of this rank's rows of one weight (the buffer's unpacked view)."""
        t = self.weights[(layer, name)]
        out = np.empty(t.ne[1] * row_bytes_q4k(t.ne[0]), np.uint8)
        self.buf.get(t, out.ctypes.data, 0, out.nbytes)
        return out

    def check(self, O) -> dict:
        """The last step's outputs of layers 0 and 1 (the two distinct weight
        sets, and the down -> q/k/v hand-over between layers) against the
        oracle on their actual inputs, this rank's rows; then the lm_head node
        once more on layer 1's output, against the oracle.  (The step is
        matmuls only, with no normalisation between layers: each layer scales
        the activations by about 20, so the deep layers' values leave the F32
        range and carry inf / NaN, which the kernels propagate.)"""
        nt = os.cpu_count() or 8
        worst = {"cos": 1.0, "maxabs_rel": 0.0}
        nodes = 0
        raw_cache = {}
        for layer in range(min(2, self.layers)):
            a = {k: v.cpu().numpy() for k, v in self.acts[layer].items()}
            a["h"] = self.h[layer].cpu().numpy()
            a["down"] = self.h[layer + 1].cpu().numpy()
            for name, N, K in LAYER_MATS:
                src = {"q": "h", "k": "h", "v": "h", "o": "q", "gate": "o", "up": "o", "down": "gate"}[name]
                key = self.weight_key(layer, name)
                if key not in raw_cache:
                    raw_cache[key] = self.raw_weights(layer, name)
                r0, nr = self.G.shard_rows(N, self.world, self.rank)
                ref = O.gemv(O.Q4_K, raw_cache[key], nr, K, a[src], nthreads=nt)
                s = O.stats(a[name][r0:r0 + nr], ref)
                worst["cos"] = min(worst["cos"], s["cos"])
                worst["maxabs_rel"] = max(worst["maxabs_rel"], s["maxabs_rel"])
                nodes += 1
        raw_cache.clear()
        x = self.h[min(2, self.layers)]
        node = self._node(self.layers, "lm_head", self._vec(x.data_ptr(), HIDDEN), self.logits.data_ptr(), VOCAB)
        if not self.be.compute([node]):
            raise RuntimeError(f"compute_graph (lm_head check) failed: {self.G.last_error()}")
        self.be.synchronize()
        r0, nr = self.G.shard_rows(VOCAB, self.world, self.rank)
        ref = O.gemv(O.Q4_K, self.raw_weights(self.layers, "lm_head"), nr, HIDDEN, x.cpu().numpy(), nthreads=nt)
        s = O.stats(self.logits.cpu().numpy()[r0:r0 + nr], ref)
        worst["cos"] = min(worst["cos"], s["cos"])
        worst["maxabs_rel"] = max(worst["maxabs_rel"], s["maxabs_rel"])
        return {"nodes": nodes + 1, **worst}


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

    plan = []  # (weights, outputs, x, K) per launch
    groups = [(("q", "k", "v"), "h"), (("o",), "q"), (("gate", "up"), "o"), (("down",), "gate")]
    for layer in range(model.layers):
        a = dict(model.acts[layer], h=model.h[layer], down=model.h[layer + 1])
        for names, x in groups:
            ws = [model.weights[(layer, n)] for n in names]
            plan.append(([w.data for w in ws], [a[n].data_ptr() for n in names], [w.ne[1] for w in ws],
                         a[x].data_ptr(), ws[0].ne[0]))
    w = model.weights[(model.layers, "lm_head")]
    plan.append(([w.data], [model.logits.data_ptr()], [w.ne[1]], model.h[model.layers].data_ptr(), HIDDEN))
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


# ---------------------------------------------- per-format GEMV (configs[0-2])
PER_FORMAT = ([("Q4_0", 4096, 4096), ("Q4_0", 8192, 8192), ("Q4_0", 17408, 5120)]
              + [(name, n, k) for name in ("Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ2_S", "IQ3_S", "IQ3_XXS", "IQ4_XS")
                 for n, k in ((11008, 2048), (2048, 11008 // 256 * 256))])


def per_format_sweep(torch, G, O, iters: int = 200, cpu_seconds: float = 0.4) -> list[dict]:
    """Every claimed format at the BASELINE configs[0-2] shapes (K of the
    256-value formats rounded down to a block multiple: 2048 x 10752).
    Weights N(0, 0.02) quantised by the oracle (the ggml reference
    quantisers' algorithms), x ~ N(0, 1).  GPU: b200_gemv launched as one CUDA
    graph of `iters` launches rotating through copies of the weights past
    twice the L2, CUDA events on the stream; one output checked against the
    oracle.  CPU: the reference's own engine (XdnaGemvEngine::run / run_quant,
    its OpenMP threads) where it implements the format, else the oracle port
    on every host thread."""
    peak, _ = measured_peak()
    ref_engine = O.RefEngine() if O.ref_available() else None
    nt = os.cpu_count() or 8
    out = []
    for name, n, k in PER_FORMAT:
        t = G.CLAIMED[name]
        rng = np.random.default_rng(zlib.crc32(f"{name}:{n}:{k}".encode()))
        raw = O.quantize(t, rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32), nthreads=nt)
        x = rng.normal(0.0, 1.0, k).astype(np.float32)
        nbytes = raw.nbytes
        copies = max(2, -(-2 * L2_BYTES // nbytes))
        s = torch.cuda.Stream()
        sh = s.cuda_stream
        with torch.cuda.stream(s):
            d_raw = torch.from_numpy(raw).cuda()
            pk = torch.empty_like(d_raw)
            G.check(G.lib().b200_repack(t, d_raw.data_ptr(), pk.data_ptr(), n, k, sh), "repack")
            ws = [pk] + [pk.clone() for _ in range(copies - 1)]
            d_x = torch.from_numpy(x).cuda()
            d_y = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        L = G.lib()

        def launch(i: int) -> None:
            G.check(L.b200_gemv(t, ws[i % copies].data_ptr(), d_x.data_ptr(), d_y.data_ptr(), n, k, sh, 1), "gemv")

        for i in range(5):
            launch(i)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(iters):
                launch(i)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            g.replay()
            e0.record(s)
            g.replay()
            e1.record(s)
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / iters
        gbs = nbytes / (us * 1e-6) / 1e9
        chk = parity(O, d_y.cpu().numpy(), O.gemv(t, raw, n, k, x, nthreads=nt))
        del g, ws, pk, d_raw
        # the reference's CPU engine on the same bytes
        y = np.empty(n, np.float32)
        if ref_engine is not None and t in O.REF_TYPES:
            kind, cores = "reference", 4 if t == O.Q4_0 else 8  # Q4GemvEngine: 4 threads; run_quant: 8

            def cpu_call():
                ref_engine.run(t, raw, n, k, x, y)
        else:
            kind, cores = "port", nt

            def cpu_call():
                y[:] = O.gemv(t, raw, n, k, x, nthreads=nt)
        cpu_call()
        m, c0 = 0, time.perf_counter()
        while True:
            cpu_call()
            m += 1
            el = time.perf_counter() - c0
            if el >= cpu_seconds:
                break
        out.append({"type": name, "n": n, "k": k, "weight_bytes": nbytes, "us": round(us, 2), "gb_s": round(gbs, 1),
                    "frac_of_measured": round(gbs / peak, 4), "pct_of_8tbs": round(100.0 * gbs / NOMINAL_HBM_GBS, 1),
                    "cos": chk["cos"], "maxabs_rel": chk["maxabs_rel"], "parity_ok": chk["ok"],
                    "cpu_gb_s": round(m * nbytes / el / 1e9, 2), "cpu_kind": kind, "cpu_cores": cores})
    if ref_engine is not None:
        ref_engine.close()
    return out


# ------------------------------------------- Qwen2.5-3B-shaped decode
def qwen3b_decode(torch, G, O, be, n_new: int = 128, n_check: int = 32) -> dict:
    """BASELINE configs[3] through xdna.cpp_b200/decode_harness.py: 16 seeded
    prompt tokens and n_new greedy tokens with every M = 1 MUL_MAT on the
    plugin (host activations) and the other ops on the host; tok/s over all
    16 + n_new steps, then the first n_check tokens against the same decode
    driven by the oracle's matmuls on the same weight bytes."""
    import decode_harness as D

    cfg, seed = D.QWEN25_3B, 3
    prompt = D.prompt_ids(cfg, seed, 16)
    shapes = D.mat_shapes(cfg)
    m = D.PluginModel(torch, be, cfg, seed)
    try:
        dec = D.Decoder(cfg, seed, m.matmul)
        t0 = time.perf_counter()
        toks, _ = dec.generate(prompt, n_new)
        el = time.perf_counter() - t0
        raws = {k: m.raw(k) for k in D.weight_keys(cfg)}
    finally:
        m.free()
    nt = os.cpu_count() or 8

    def mm_oracle(keys, x):
        return [O.gemv(O.Q4_0, raws[k], shapes[k[1]][0], shapes[k[1]][1], np.ascontiguousarray(x), nthreads=nt)
                for k in keys]

    toks_ref, _ = D.Decoder(cfg, seed, mm_oracle).generate(prompt, n_check)
    match = sum(1 for a, b in zip(toks[:n_check], toks_ref) if a == b)
    return {"tok_s": round((16 + n_new) / el, 2), "steps": 16 + n_new, "seconds": round(el, 2),
            "greedy_match": f"{match}/{n_check}", "match_ok": match == n_check,
            "path": "decode_harness.py: host RMSNorm/RoPE/attention/SwiGLU in numpy, 253 MUL_MATs per token "
                    "through ggml_backend_xdna_compute_graph with host activations",
            "weight_bytes_per_token": sum(shapes[n][0] * G.row_bytes(G.Q4_0, shapes[n][1])
                                          for _, n in D.weight_keys(cfg))}


def run_b200_arm(args, dist: Dist) -> None:
    import torch

    import ggml_b200 as G

    G.lib()
    torch.cuda.set_device(dist.local_rank)
    t_setup = time.perf_counter()
    nccl_id = dist.broadcast_bytes(G.nccl_unique_id() if dist.rank == 0 else None) if dist.world > 1 else None
    be = G.Backend(dist.local_rank, dist.world, dist.rank, nccl_id)
    model = Model(G, torch, be, dist.world, dist.rank, layers=args.layers)
    torch.cuda.synchronize()
    setup_s = time.perf_counter() - t_setup
    wbt = weight_bytes_per_token(args.layers)
    dist.barrier()

    for _ in range(args.warmup):
        if not be.compute(model.nodes):
            raise RuntimeError(f"compute_graph failed: {G.last_error()}")
    be.synchronize()
    dist.barrier()
    pad = 0.0 if args.profile_run else 1.0
    with ClockSampler(dist.local_rank) as clk:
        # the sampler needs a moment to start: keep the GPU busy with untimed
        # steps for about a second before the timed ones and after them
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < pad:
            be.compute(model.nodes)
        be.synchronize()
        ms = time_steps(torch, be, model.nodes, args.steps)
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < pad / 2:
            be.compute(model.nodes)
        be.synchronize()
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

    # the timed step's outputs against the oracle (one more device-resident
    # step, so the per-layer activations hold a step of the timed node list)
    O = oracle_module()
    chk = {"nodes": 0, "cos": 1.0, "maxabs_rel": 0.0}
    if not args.profile_run:
        if not be.compute(model.nodes):
            raise RuntimeError(f"compute_graph failed: {G.last_error()}")
        be.synchronize()
        chk = model.check(O)
    chk["cos"] = dist.reduce(chk["cos"], "min")
    chk["maxabs_rel"] = dist.max(chk["maxabs_rel"])
    chk["ok"] = bool(chk["cos"] >= COS_MIN and chk["maxabs_rel"] <= MAXABS_REL)
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
    ratio, traffic_src = profiled_traffic_ratio()
    traffic = int(round(ratio * model.local_bytes)) if ratio else None
    achieved = model.local_bytes / (k_ms * 1e-3) / 1e9

    cpu, per_fmt, qwen = None, None, None
    if dist.rank == 0 and dist.world == 1 and not args.profile_run:
        cpu = reference_cpu_sample(seconds=args.cpu_seconds)
        per_fmt = per_format_sweep(torch, G, O)
        qwen = qwen3b_decode(torch, G, O, be)
    dist.barrier()

    if dist.rank == 0:
        value = wbt / (ms_step * 1e-3) / 1e9
        e2e_gbs = wbt / (e2e_ms * 1e-3) / 1e9
        nl = launches_per_token(args.layers)
        config = {
            "workload": f"llama3-70b-shaped Q4_K decode: {args.layers * 7 + 1} M=1 MUL_MATs per token "
                        f"({args.layers} layers x q,k,v,o,gate,up,down + lm_head), rows sharded over N GPUs, outputs "
                        "exchanged over NVLink by the GEMV and a gather kernel (NCCL all-gather fallback)",
            "weight_bytes_per_token": wbt, "matmuls_per_token": args.layers * 7 + 1,
            "batch": 1, "parallelism": f"rows{dist.world}",
            "tok_s": round(1000.0 / ms_step, 3),
            "pct_of_8tbs": round(100.0 * value / (NOMINAL_HBM_GBS * dist.world), 2),
            "l2": "per-step weights (39 GB) exceed the 126 MB L2; no flush needed",
            "setup_s": round(setup_s, 1),
        }
        if per_fmt is not None:
            config["per_format"] = per_fmt
        if qwen is not None:
            config["qwen3b_decode"] = qwen
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: random-init N(0,0.02) weights quantised on the GPU to Q4_K, N(0,1) activations",
            "config": config,
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "tok_s": round(1000.0 / e2e_ms, 3),
                    "h2d_bytes_per_step": HIDDEN * 4, "d2h_bytes_per_step": VOCAB * 4,
                    "path": "ggml_backend_xdna_compute_graph, token input from pinned host memory, logits to host"},
            "check": {"against": "CPU oracle (oracle/quant_oracle.c) on each node's actual input, this rank's rows",
                      "nodes": chk["nodes"], "layers": list(range(min(2, args.layers))),
                      "lm_head_input": "layer 1's output (a separate lm_head call)", "cos_min": round(chk["cos"], 9),
                      "maxabs_rel_max": float(f"{chk['maxabs_rel']:.3e}"), "ok": chk["ok"]},
            "roofline": {"bound": "hbm", "kernel": "gemv_mma_kernel<12> (Q4_K)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": traffic, "traffic_unit": "DRAM bytes per step (all GEMV launches)",
                         "traffic_source": (f"{traffic_src}: DRAM bytes per algorithmic byte of a two-layer "
                                            "capture, times this step's algorithmic bytes") if ratio else traffic_src,
                         "algorithmic_bytes_per_step": model.local_bytes,
                         "per_launch_note": f"{nl} GEMV launches per step (q/k/v and gate/up fused); achieved = local "
                         "weight bytes per step / device time per step of " + k_src},
            "clocks": dict(clk.summary(), window="about 1 s of untimed steps, the timed steps, 0.5 s of untimed steps"),
            # one GPU: the GEMV launches + one xprep_kernel per step (every
            # later launch's x is prepared by the launch before it); N GPUs:
            # also one xchg_gather_kernel per launch (it prepares the next
            # launch's x); NCCL's kernels, on the fallback path, not counted
            "gpu_launches": args.steps * (nl * (1 if dist.world == 1 else 2) + 1),
        }
        if cpu is not None:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    be.close()
    model.buf.free()
    failed = not chk["ok"]
    if per_fmt is not None:
        failed |= not all(r["parity_ok"] for r in per_fmt)
    if qwen is not None:
        failed |= not qwen["match_ok"]
    if failed:
        raise SystemExit("bench: the outputs missed the parity bar (see the check / per_format / qwen3b_decode keys)")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers of the 70B-shaped stack (80 = the config; fewer only for profiling captures)")
    ap.add_argument("--profile-run", action="store_true",
                    help="for profiler captures: skip the CPU baseline, the per-format sweep, the Qwen-3B decode, "
                         "the untimed steps around the timed ones and the output check")
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
