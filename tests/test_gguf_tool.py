"""The GGUF per-tensor tool (xdna.cpp_b200/gguf_bench.py) on a small synthetic
GGUF file written with the gguf package: the loader finds exactly the claimed
2-D tensors with the right shapes and bytes (CPU), and the GPU run of each
matches the float64 product of the gguf-dequantised weights (GPU)."""
from __future__ import annotations

import numpy as np
import pytest

from helpers import COS_MIN, MAXABS_REL, normal_weights


def write_model(path, O):
    import gguf

    w = gguf.GGUFWriter(str(path), "llama")
    specs = [("blk.0.attn_q.weight", O.Q4_K, 64, 512), ("blk.0.ffn_down.weight", O.Q6_K, 48, 1024),
             ("blk.0.attn_k.weight", O.Q4_0, 32, 256), ("blk.0.ffn_up.weight", O.IQ4_XS, 32, 512)]
    out = {}
    for i, (name, t, N, K) in enumerate(specs):
        raw = O.quantize(t, normal_weights(N, K, seed=900 + i)).reshape(N, -1)
        w.add_tensor(name, raw, raw_dtype=gguf.GGMLQuantizationType(t))
        out[name] = (t, N, K, raw.reshape(-1))
    w.add_tensor("output_norm.weight", np.ones(512, np.float32))  # unclaimed (F32)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return out


def test_loader_finds_claimed_tensors(G, O, tmp_path):
    import gguf_bench as GB

    path = tmp_path / "m.gguf"
    want = write_model(path, O)
    got = {name: (t, N, K, raw) for name, t, N, K, raw in GB.claimed_tensors(str(path))}
    assert set(got) == set(want)
    for name, (t, N, K, raw) in want.items():
        gt, gN, gK, graw = got[name]
        assert (gt, gN, gK) == (t, N, K)
        np.testing.assert_array_equal(graw, raw)


@pytest.mark.gpu
def test_gguf_tensors_on_gpu(cuda, G, O, tmp_path):
    import gguf_bench as GB

    path = tmp_path / "m.gguf"
    write_model(path, O)
    with G.Backend(0) as be:
        for name, t, N, K, raw in GB.claimed_tensors(str(path)):
            r = GB.bench_tensor(cuda, be, name, t, N, K, raw, iters=3, check_bytes=1 << 30)
            assert r["claimed"] and r["gb_s"] > 0, r
            assert r["cos"] >= COS_MIN and r["maxabs_rel"] <= MAXABS_REL * 10, r
