#!/usr/bin/env python
"""Greedy decode of a random-init Qwen2.5-3B-shaped model with every M = 1
MUL_MAT offloaded to the B200 plugin.

This stands in for llama.cpp when only MUL_MAT is claimed by the plugin
(src/ggml-xdna.cpp:95-147 claims MUL_MAT alone): the token embedding, RMSNorm,
RoPE, grouped-query attention, SwiGLU and the residual adds run on the host in
float32, and each matmul goes through ggml_backend_xdna_compute_graph with
host activations, as ggml's scheduler would hand them over.  The matmul is a
parameter of the decoder, so the same host arithmetic can be driven by
another implementation of the matmuls (the tests drive it with the CPU
oracle) and the greedy tokens compared.

Model (Qwen2.5-3B shapes): hidden 2048, 36 layers, 16 query / 2 KV heads of
128, SwiGLU intermediate 11008, vocab 151936, RMSNorm eps 1e-6, RoPE theta
1e6.  Random init: every linear weight N(0, 0.02), drawn and quantised to
Q4_0 on the GPU (b200_fill_normal + b200_quantize) and uploaded into a B200
buffer; embedding rows N(0, 0.02) drawn on the host per token id from a
seeded generator; norm weights 1; no biases; lm_head untied.  253 MUL_MATs
(1,735,704,576 weight bytes) per token.

Usage: python xdna.cpp_b200/decode_harness.py [--layers 36] [--prompt 16] [--new 128] [--seed 3]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys
import time
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import ggml_b200 as G  # noqa: E402

QWEN25_3B = dict(hidden=2048, layers=36, heads=16, kv_heads=2, head_dim=128, inter=11008, vocab=151936,
                 theta=1.0e6, eps=1.0e-6)
LAYER_MATS = ("q", "k", "v", "o", "gate", "up", "down")


def mat_shapes(cfg: dict) -> dict:
    """(N, K) of each linear weight name."""
    h, kv, d, f = cfg["hidden"], cfg["kv_heads"] * cfg["head_dim"], cfg["heads"] * cfg["head_dim"], cfg["inter"]
    return {"q": (d, h), "k": (kv, h), "v": (kv, h), "o": (h, d), "gate": (f, h), "up": (f, h), "down": (h, f),
            "lm_head": (cfg["vocab"], h)}


def weight_keys(cfg: dict) -> list[tuple[int, str]]:
    return [(layer, n) for layer in range(cfg["layers"]) for n in LAYER_MATS] + [(cfg["layers"], "lm_head")]


def embedding_row(cfg: dict, seed: int, token: int) -> np.ndarray:
    rng = np.random.default_rng([seed, 7, token])
    return rng.normal(0.0, 0.02, cfg["hidden"]).astype(np.float32)


def prompt_ids(cfg: dict, seed: int, n: int) -> list[int]:
    return [int(t) for t in np.random.default_rng([seed, 11]).integers(0, cfg["vocab"], n)]


class Decoder:
    """Host side of the decode.  matmul(keys, x) returns W_key @ x for each
    (layer, name) key of a group that shares x (q/k/v, gate/up, or one)."""

    def __init__(self, cfg: dict, seed: int, matmul):
        self.cfg, self.seed, self.matmul = cfg, seed, matmul
        hd = cfg["head_dim"]
        self.inv_freq = (cfg["theta"] ** (-np.arange(0, hd, 2, dtype=np.float64) / hd)).astype(np.float64)
        self.kcache = [[] for _ in range(cfg["layers"])]
        self.vcache = [[] for _ in range(cfg["layers"])]

    def rmsnorm(self, x: np.ndarray) -> np.ndarray:
        return (x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + self.cfg["eps"])).astype(np.float32)

    def rope(self, v: np.ndarray, nheads: int, pos: int) -> np.ndarray:
        hd = self.cfg["head_dim"]
        a = pos * self.inv_freq
        cos, sin = np.cos(a).astype(np.float32), np.sin(a).astype(np.float32)
        v = v.reshape(nheads, hd)
        x1, x2 = v[:, : hd // 2], v[:, hd // 2:]  # rotate-half pairing (i, i + hd/2)
        return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=1)

    def step(self, token: int, pos: int) -> np.ndarray:
        cfg = self.cfg
        H, KVH, hd = cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
        x = embedding_row(cfg, self.seed, token)
        for layer in range(cfg["layers"]):
            h = self.rmsnorm(x)
            q, k, v = self.matmul([(layer, "q"), (layer, "k"), (layer, "v")], h)
            q = self.rope(q, H, pos)
            self.kcache[layer].append(self.rope(k, KVH, pos))
            self.vcache[layer].append(v.reshape(KVH, hd))
            K = np.stack(self.kcache[layer])  # [T, KVH, hd]
            V = np.stack(self.vcache[layer])
            att = np.empty((H, hd), np.float32)
            for head in range(H):
                g = head // (H // KVH)
                s = (K[:, g, :] @ q[head]) / np.float32(np.sqrt(hd))
                p = np.exp(s - s.max())
                att[head] = (p / p.sum()) @ V[:, g, :]
            (o,) = self.matmul([(layer, "o")], att.reshape(-1))
            x = x + o
            h2 = self.rmsnorm(x)
            gate, up = self.matmul([(layer, "gate"), (layer, "up")], h2)
            a = (gate / (1.0 + np.exp(-gate)) * up).astype(np.float32)
            (d,) = self.matmul([(layer, "down")], a)
            x = x + d
        (logits,) = self.matmul([(cfg["layers"], "lm_head")], self.rmsnorm(x))
        return logits

    def generate(self, prompt: list[int], n_new: int):
        """Feeds the prompt one token at a time (M = 1), then decodes n_new
        tokens greedily.  Returns the generated tokens and each step's logits."""
        tokens, logits_all = [], []
        pos, tok = 0, None
        for t in prompt:
            logits = self.step(t, pos)
            pos += 1
        for _ in range(n_new):
            tok = int(np.argmax(logits))
            tokens.append(tok)
            logits_all.append(logits)
            logits = self.step(tok, pos)
            pos += 1
        return tokens, logits_all


class PluginModel:
    """The model's Q4_0 weights in one B200 buffer, and the matmul through
    ggml_backend_xdna_compute_graph (host activations)."""

    def __init__(self, torch, be, cfg: dict, seed: int):
        self.cfg, self.be = cfg, be
        shapes = mat_shapes(cfg)
        keys = weight_keys(cfg)
        total = sum(shapes[n][0] * G.row_bytes(G.Q4_0, shapes[n][1]) for _, n in keys)
        self.buf = G.Buffer(total + 4096 * (len(keys) + 2), dev=be.dev)
        self.w = {}
        L = G.lib()
        for layer, name in keys:
            N, K = shapes[name]
            t = self.buf.alloc(G.tensor(G.Q4_0, [K, N, 1, 1], name=f"{name}.{layer}"))
            w = torch.empty(N * K, dtype=torch.float32, device="cuda")
            G.check(L.b200_fill_normal(w.data_ptr(), w.numel(), zlib.crc32(f"{seed}:{layer}:{name}".encode()),
                                       0.02, 0), "fill_normal")
            q = torch.empty(N * G.row_bytes(G.Q4_0, K), dtype=torch.uint8, device="cuda")
            G.check(L.b200_quantize(G.Q4_0, w.data_ptr(), q.data_ptr(), N, K, 0), "quantize")
            torch.cuda.synchronize()
            self.buf.set_device(t, q.data_ptr(), 0, q.numel())
            self.w[(layer, name)] = (t, N, K)
        self._keep = []

    def raw(self, key) -> np.ndarray:
        """GGUF bytes of one weight (the unpacked view of the buffer)."""
        t, N, K = self.w[key]
        out = np.empty(N * G.row_bytes(G.Q4_0, K), np.uint8)
        self.buf.get(t, out.ctypes.data, 0, out.nbytes)
        return out

    def matmul(self, keys, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        ys, nodes = [], []
        for key in keys:
            t, N, K = self.w[key]
            y = np.empty(N, np.float32)
            xt = G.tensor(G.F32, [K, 1, 1, 1], data=x.ctypes.data)
            nodes.append(G.mul_mat_node(t, xt, y.ctypes.data, N, name=f"{key[1]}.{key[0]}"))
            ys.append(y)
            self._keep.append(xt)
        if not self.be.compute(nodes):
            raise RuntimeError(f"compute_graph failed: {G.last_error()}")
        self._keep.clear()
        return ys

    def free(self) -> None:
        self.buf.free()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--layers", type=int, default=QWEN25_3B["layers"])
    ap.add_argument("--prompt", type=int, default=16)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--seed", type=int, default=3)
    ap.add_argument("--device", type=int, default=0)
    a = ap.parse_args()
    import torch

    if not torch.cuda.is_available():
        sys.exit("decode_harness needs a CUDA device")
    torch.cuda.set_device(a.device)
    cfg = dict(QWEN25_3B, layers=a.layers)
    with G.Backend(a.device) as be:
        m = PluginModel(torch, be, cfg, a.seed)
        dec = Decoder(cfg, a.seed, m.matmul)
        t0 = time.perf_counter()
        toks, _ = dec.generate(prompt_ids(cfg, a.seed, a.prompt), a.new)
        el = time.perf_counter() - t0
        m.free()
    steps = a.prompt + a.new
    print(json.dumps({"model": "qwen2.5-3b-shaped Q4_0 (random init)", "layers": cfg["layers"], "prompt": a.prompt,
                      "new_tokens": a.new, "tok_s": round(steps / el, 2), "tokens": toks[:32]}))


if __name__ == "__main__":
    main()
