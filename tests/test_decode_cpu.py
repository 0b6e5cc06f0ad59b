"""The decode harness (xdna.cpp_b200/decode_harness.py) on a tiny
Qwen2-style config, on the CPU: driven once by the oracle's Q4_0 matmul and
once by a float64 product of the gguf-dequantised weights (a second,
independent implementation), it must produce the same greedy tokens, with
per-step logits that agree closely.  This checks the harness's host
arithmetic (RMSNorm, RoPE, grouped-query attention, SwiGLU) and its greedy
loop; the GPU test drives the same harness with the plugin."""
from __future__ import annotations

import numpy as np

from helpers import normal_weights

TINY = dict(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, inter=512, vocab=1000, theta=1.0e6, eps=1.0e-6)


def test_harness_greedy_decode_two_matmul_paths_agree(O):
    import gguf
    from gguf.quants import dequantize

    import decode_harness as D

    shapes = D.mat_shapes(TINY)
    raws, deq = {}, {}
    for i, (layer, name) in enumerate(D.weight_keys(TINY)):
        N, K = shapes[name]
        raws[(layer, name)] = O.quantize(O.Q4_0, normal_weights(N, K, seed=500 + i), nthreads=4)
        deq[(layer, name)] = dequantize(raws[(layer, name)].reshape(N, -1), gguf.GGMLQuantizationType.Q4_0).astype(
            np.float64).reshape(N, K)

    def mm_oracle(keys, x):
        return [O.gemv(O.Q4_0, raws[k], shapes[k[1]][0], shapes[k[1]][1], np.ascontiguousarray(x), nthreads=4)
                for k in keys]

    def mm_f64(keys, x):
        return [(deq[k] @ x.astype(np.float64)).astype(np.float32) for k in keys]

    prompt = D.prompt_ids(TINY, 5, 6)
    t1, l1 = D.Decoder(TINY, 5, mm_oracle).generate(prompt, 10)
    t2, l2 = D.Decoder(TINY, 5, mm_f64).generate(prompt, 10)
    assert t1 == t2
    for a, b in zip(l1, l2):
        cos = float(a.astype(np.float64) @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
        assert cos >= 0.99999, cos
