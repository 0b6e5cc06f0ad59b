"""greedy decode of a random-init Qwen2.5-3B-shaped
model (36 layers, all linear weights Q4_0) with every M = 1 MUL_MAT offloaded
to the B200 plugin through compute_graph and the other ops on the host
(xdna.cpp_b200/decode_harness.py).  The reference for the greedy tokens is
the same harness with the CPU oracle's matmuls on the same weight bytes (the
stand-in for llama.cpp's CPU backend, which is not available here): 16 prompt
tokens, then 32 decode steps with identical tokens and logits that agree."""
from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_qwen3b_greedy_decode_matches_oracle(cuda, G, O):
    import decode_harness as D

    cfg, seed = D.QWEN25_3B, 3
    prompt = D.prompt_ids(cfg, seed, 16)
    shapes = D.mat_shapes(cfg)
    with G.Backend(0) as be:
        m = D.PluginModel(cuda, be, cfg, seed)
        toks_gpu, logits_gpu = D.Decoder(cfg, seed, m.matmul).generate(prompt, 32)
        raws = {k: m.raw(k) for k in D.weight_keys(cfg)}
        m.free()
    nt = os.cpu_count() or 8

    def mm_oracle(keys, x):
        return [O.gemv(O.Q4_0, raws[k], shapes[k[1]][0], shapes[k[1]][1], np.ascontiguousarray(x), nthreads=nt)
                for k in keys]

    toks_ref, logits_ref = D.Decoder(cfg, seed, mm_oracle).generate(prompt, 32)
    assert toks_gpu == toks_ref, (toks_gpu, toks_ref)
    for i, (a, b) in enumerate(zip(logits_gpu, logits_ref)):
        cos = float(a.astype(np.float64) @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
        rel = float(np.abs(a - b).max() / np.abs(b).max())
        assert cos >= 0.99999 and rel <= 1e-3, (i, cos, rel)
