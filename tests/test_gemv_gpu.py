"""GPU parity tests of the decode-GEMV kernels, through the C ABI.

Each case quantises seeded inputs, runs the sm_100a kernel and compares it with
the CPU oracle (the reference's scalar arithmetic restated in
oracle/quant_oracle.c), at the bar of BASELINE.json: cos >= 0.999999 and
max-abs error <= 1e-4 * max|y|.  The test intents follow the reference's own
suites: tests/test-gemv-accuracy.cpp (accuracy, zero invariance, boundary N,
model shapes, K validation, concurrency) and tests/test-kquants-gemv.cpp
(per-type accuracy, zero invariance, shape sweep).
"""
import ctypes as C
import os
import threading

import numpy as np
import pytest

from helpers import check_parity, gemv_gpu, normal_weights, normal_x, random_blocks, to_dev

pytestmark = pytest.mark.gpu

TYPES = ["Q4_0", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ3_XXS", "IQ3_S", "IQ2_S", "IQ4_XS"]
# (N, K): one full-tile case, odd row counts (partial last tile), an odd super-block count
SHAPES = [(64, 512), (33, 768), (127, 256), (6, 256 * 43), (1, 256)]


@pytest.mark.parametrize("name", TYPES)
@pytest.mark.parametrize("N,K", SHAPES)
def test_parity_quantized_normal(cuda, G, O, name, N, K):
    t = G.CLAIMED[name]
    W = normal_weights(N, K, seed=1000 + N + K)
    raw = O.quantize(t, W)
    x = normal_x(K, seed=7 + K)
    y = gemv_gpu(cuda, G, t, raw, N, K, x)
    check_parity(y, O.gemv(t, raw, N, K, x), f"{name} {N}x{K}")


@pytest.mark.parametrize("name", TYPES)
def test_parity_random_blocks(cuda, G, O, name):
    t = G.CLAIMED[name]
    N, K = 96, 1024
    raw = random_blocks(t, N, K, seed=101)
    x = np.random.default_rng(42).uniform(-0.5, 0.5, K).astype(np.float32)
    y = gemv_gpu(cuda, G, t, raw, N, K, x)
    check_parity(y, O.gemv(t, raw, N, K, x), name)


@pytest.mark.parametrize("name", TYPES)
def test_zero_activations_give_exact_zero(cuda, G, O, name):
    # tests/test-gemv-accuracy.cpp:184-217 and tests/test-kquants-gemv.cpp:262-270
    t = G.CLAIMED[name]
    N, K = 40, 512
    raw = random_blocks(t, N, K, seed=505)
    y = gemv_gpu(cuda, G, t, raw, N, K, np.zeros(K, np.float32))
    assert np.all(y == 0.0)


@pytest.mark.parametrize("N,K", [(1, 32), (1, 4096), (33, 64), (127, 128), (255, 64), (384, 128),
                                 (513, 64), (1536, 128), (256, 256), (1024, 1024)])
def test_q4_0_boundary_shapes(cuda, G, O, N, K):
    # tests/test-gemv-accuracy.cpp:322-371
    raw = random_blocks(G.Q4_0, N, K, seed=810)
    x = np.random.default_rng(811).uniform(-1, 1, K).astype(np.float32)
    y = gemv_gpu(cuda, G, G.Q4_0, raw, N, K, x)
    check_parity(y, O.gemv(G.Q4_0, raw, N, K, x), f"Q4_0 {N}x{K}")


@pytest.mark.parametrize("N,K", [(4096, 4096), (11008, 4096)])
def test_q4_0_model_shapes(cuda, G, O, N, K):
    # tests/test-gemv-accuracy.cpp:373-396
    raw = random_blocks(G.Q4_0, N, K, seed=820)
    x = np.random.default_rng(821).uniform(-1, 1, K).astype(np.float32)
    y = gemv_gpu(cuda, G, G.Q4_0, raw, N, K, x)
    check_parity(y, O.gemv(G.Q4_0, raw, N, K, x), f"Q4_0 {N}x{K}")


@pytest.mark.parametrize("name", TYPES)
@pytest.mark.parametrize("N,K", [(11008, 2048), (2048, 11008)])
def test_sweep_shapes_config2(cuda, G, O, name, N, K):
    # BASELINE.json configs[2] shapes, synthetic N(0, 0.02) weights, N(0, 1) x
    t = G.CLAIMED[name]
    if t == G.Q4_0:
        pytest.skip("configs[2] is the K-quant / IQ sweep")
    raw = O.quantize(t, normal_weights(N, K, seed=31))
    x = normal_x(K, seed=32)
    y = gemv_gpu(cuda, G, t, raw, N, K, x)
    check_parity(y, O.gemv(t, raw, N, K, x), f"{name} {N}x{K}")


@pytest.mark.parametrize("name", TYPES)
@pytest.mark.parametrize("N,K", [(64, 512), (37, 768), (16, 256 * 43), (48, 2048)])
def test_device_repack_matches_host_layout(cuda, G, name, N, K):
    # the GPU repack must produce exactly the layout the host reference
    # implementation of formats.cuh describes, and unpack must invert it
    t = G.CLAIMED[name]
    raw = random_blocks(t, N, K, seed=N * K)
    host = np.zeros_like(raw)
    G.check(G.lib().b200_repack_host(t, raw.ctypes.data, host.ctypes.data, N, K), "repack_host")
    d_raw = to_dev(cuda, raw)
    d_pk = cuda.zeros_like(d_raw)
    d_back = cuda.zeros_like(d_raw)
    G.check(G.lib().b200_repack(t, d_raw.data_ptr(), d_pk.data_ptr(), N, K, 0), "repack")
    G.check(G.lib().b200_unpack(t, d_pk.data_ptr(), d_back.data_ptr(), N, K, 0), "unpack")
    cuda.cuda.synchronize()
    assert np.array_equal(d_pk.cpu().numpy(), host)
    assert np.array_equal(d_back.cpu().numpy(), raw)


def test_quantizers_match_oracle(cuda, G, O):
    for t in (G.Q4_0, G.Q4_K):
        N, K = 64, 2048
        W = normal_weights(N, K, seed=77)
        d_w = to_dev(cuda, W)
        d_q = cuda.empty(N * G.row_bytes(t, K), dtype=cuda.uint8, device="cuda")
        G.check(G.lib().b200_quantize(t, d_w.data_ptr(), d_q.data_ptr(), N, K, 0), "quantize")
        cuda.cuda.synchronize()
        assert np.array_equal(d_q.cpu().numpy(), O.quantize(t, W)), G.TYPE_NAME[t]


def test_fill_normal_statistics(cuda, G):
    n = 1 << 20
    d = cuda.empty(n, dtype=cuda.float32, device="cuda")
    G.check(G.lib().b200_fill_normal(d.data_ptr(), n, 123, 0.02, 0), "fill_normal")
    a = d.cpu().numpy()
    assert np.isfinite(a).all()
    assert abs(a.mean()) < 1e-4 and abs(a.std() - 0.02) < 2e-4


def test_bf16_activation_path(cuda, G, O):
    # reference run_bf16 (src/xdna-gemv-engine.cpp:1894-1908), checked against gemv_bf16
    N, K = 512, 256
    raw = random_blocks(G.Q4_0, N, K, seed=303)
    xb = O.f32_to_bf16(np.random.default_rng(404).uniform(-1, 1, K).astype(np.float32))
    d_xb = to_dev(cuda, xb)
    d_x = cuda.empty(K, dtype=cuda.float32, device="cuda")
    G.check(G.lib().b200_bf16_to_f32(d_xb.data_ptr(), d_x.data_ptr(), K, 0), "bf16")
    cuda.cuda.synchronize()
    x = d_x.cpu().numpy()
    assert np.array_equal(x.view(np.uint32) >> 16, xb.astype(np.uint32))
    y = gemv_gpu(cuda, G, G.Q4_0, raw, N, K, x)
    check_parity(y, O.gemv_q4_0_bf16(raw, N, K, xb), "bf16")


def test_launcher_rejects_bad_shapes(cuda, G):
    L = G.lib()
    d = cuda.zeros(1024, dtype=cuda.float32, device="cuda")
    assert L.b200_gemv(G.Q4_0, d.data_ptr(), d.data_ptr(), d.data_ptr(), 10, 33, 0, 0) != 0
    assert L.b200_gemv(G.Q4_K, d.data_ptr(), d.data_ptr(), d.data_ptr(), 10, 5121, 0, 0) != 0
    assert L.b200_gemv(7, d.data_ptr(), d.data_ptr(), d.data_ptr(), 10, 256, 0, 0) != 0
    assert L.b200_gemv(G.Q4_0, d.data_ptr(), d.data_ptr() + 4, d.data_ptr(), 10, 256, 0, 0) != 0


# ------------------------------------------------------------------ compat ABI
def _np_ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def test_compute_graph_known_answer(cuda, G):
    # tests/test-backend.cpp:59-97: N=128, K=256, qs=0x99, d=1, x=0.5 -> 128.0
    N, K = 128, 256
    blk = np.zeros((N * K // 32, 18), np.uint8)
    blk[:, 0], blk[:, 1] = 0x00, 0x3C
    blk[:, 2:] = 0x99
    w_data = blk.reshape(-1).copy()
    x_data = np.full(K, 0.5, np.float32)
    y_data = np.zeros(N, np.float32)
    w = G.tensor(G.Q4_0, [K, N, 1, 1], data=_np_ptr(w_data))
    x = G.tensor(G.F32, [K, 1, 1, 1], data=_np_ptr(x_data))
    node = G.mul_mat_node(w, x, _np_ptr(y_data), N)
    with G.Backend(0) as be:
        assert G.lib().ggml_backend_is_xdna(be.h)
        assert be.compute([node])
    assert np.all(np.abs(y_data - 128.0) < 1e-3)


def test_compute_graph_host_and_device_operands(cuda, G, O):
    N, K = 256, 2048
    t = G.Q4_K
    raw = O.quantize(t, normal_weights(N, K, seed=5))
    x = normal_x(K, seed=6)
    y_ref = O.gemv(t, raw, N, K, x)
    with G.Backend(0) as be:
        # (a) everything in host memory: weights uploaded per call
        y = np.zeros(N, np.float32)
        w = G.tensor(t, [K, N, 1, 1], data=_np_ptr(raw))
        xt = G.tensor(G.F32, [K, 1, 1, 1], data=_np_ptr(x))
        assert be.compute([G.mul_mat_node(w, xt, _np_ptr(y), N)])
        check_parity(y, y_ref, "host operands")
        # (b) weights resident in a B200 buffer, x / y in device memory
        buf = G.Buffer(raw.nbytes + 8192, dev=0)
        wd = buf.alloc(G.tensor(t, [K, N, 1, 1]))
        buf.set(wd, _np_ptr(raw), 0, raw.nbytes)
        d_x = to_dev(cuda, x)
        d_y = cuda.zeros(N, dtype=cuda.float32, device="cuda")
        xt2 = G.tensor(G.F32, [K, 1, 1, 1], data=d_x.data_ptr())
        assert be.compute([G.mul_mat_node(wd, xt2, d_y.data_ptr(), N)])
        check_parity(d_y.cpu().numpy(), y_ref, "device operands")
        # (c) resident weights, host x / y
        y2 = np.zeros(N, np.float32)
        assert be.compute([G.mul_mat_node(wd, xt, _np_ptr(y2), N)])
        check_parity(y2, y_ref, "resident weights, host activations")
        buf.free()


def test_compute_graph_chained_host_nodes(cuda, G, O):
    # node 2 consumes node 1's host output inside one compute_graph call
    t = G.Q4_0
    K = N = 512
    r1 = O.quantize(t, normal_weights(N, K, seed=1))
    r2 = O.quantize(t, normal_weights(N, K, seed=2))
    x = normal_x(K, seed=3)
    h = np.zeros(N, np.float32)
    y = np.zeros(N, np.float32)
    w1 = G.tensor(t, [K, N, 1, 1], data=_np_ptr(r1))
    w2 = G.tensor(t, [K, N, 1, 1], data=_np_ptr(r2))
    xt = G.tensor(G.F32, [K, 1, 1, 1], data=_np_ptr(x))
    ht = G.tensor(G.F32, [K, 1, 1, 1], data=_np_ptr(h))
    n1 = G.mul_mat_node(w1, xt, _np_ptr(h), N)
    n2 = G.mul_mat_node(w2, ht, _np_ptr(y), N)
    with G.Backend(0) as be:
        assert be.compute([n1, n2])
    h_ref = O.gemv(t, r1, N, K, x)
    check_parity(h, h_ref, "node 1")
    check_parity(y, O.gemv(t, r2, N, K, h), "node 2 (consumes node 1)")


def test_compute_graph_rejects_bad_nodes(cuda, G):
    K, N = 5121, 64
    w_data = np.zeros(64 * 1024, np.uint8)
    x_data = np.zeros(K, np.float32)
    y_data = np.zeros(N, np.float32)
    w = G.tensor(G.Q4_K, [K, N, 1, 1], data=_np_ptr(w_data))
    x = G.tensor(G.F32, [K, 1, 1, 1], data=_np_ptr(x_data))
    with G.Backend(0) as be:
        assert not be.compute([G.mul_mat_node(w, x, _np_ptr(y_data), N)])
        w.type = G.F32  # unsupported weight type
        w.ne[0] = 256
        assert not be.compute([G.mul_mat_node(w, x, _np_ptr(y_data), N)])


@pytest.mark.parametrize("N", [37, 64])  # stripe tiles; the MMA layout (N % 16 == 0)
def test_buffer_roundtrip_and_partial_writes(cuda, G, O, N):
    rng = np.random.default_rng(9)
    for name in TYPES:
        t = G.CLAIMED[name]
        K = 512
        raw = random_blocks(t, N, K, seed=11)
        buf = G.Buffer(2 * raw.nbytes + 8192, dev=0)
        wt = buf.alloc(G.tensor(t, [K, N, 1, 1]))
        buf.set(wt, _np_ptr(raw), 0, raw.nbytes)
        back = np.zeros_like(raw)
        buf.get(wt, _np_ptr(back), 0, raw.nbytes)
        assert np.array_equal(back, raw), name
        # partial, unaligned write and read
        patch = rng.integers(0, 256, 333, dtype=np.uint8)
        off = 1111
        buf.set(wt, _np_ptr(patch), off, patch.size)
        raw2 = raw.copy()
        raw2[off:off + patch.size] = patch
        part = np.zeros(500, np.uint8)
        buf.get(wt, _np_ptr(part), 1000, 500)
        assert np.array_equal(part, raw2[1000:1500]), name
        buf.get(wt, _np_ptr(back), 0, raw.nbytes)
        assert np.array_equal(back, raw2), name
        # memset and clear act on the GGUF view
        buf.memset(wt, 0x5A, 100, 700)
        raw2[100:800] = 0x5A
        buf.get(wt, _np_ptr(back), 0, raw.nbytes)
        assert np.array_equal(back, raw2), name
        for v in (0x00, 0x5A):  # 0x5A: unequal nibbles and bit pairs
            buf.clear(v)
            buf.get(wt, _np_ptr(back), 0, raw.nbytes)
            assert np.all(back == v), (name, v)
        buf.free()


def test_concurrent_threads_share_a_backend(cuda, G, O):
    # tests/test-gemv-accuracy.cpp:529-621: 4 threads x iterations, no races,
    # no cross-contamination between threads' activations
    N, K = 512, 256
    raw = random_blocks(G.Q4_0, N, K, seed=9999)
    expected = [O.gemv(G.Q4_0, raw, N, K, np.full(K, t + 1.0, np.float32)) for t in range(4)]
    errors = []
    with G.Backend(0) as be:
        def worker(tid):
            x = np.full(K, tid + 1.0, np.float32)
            y = np.zeros(N, np.float32)
            w = G.tensor(G.Q4_0, [K, N, 1, 1], data=_np_ptr(raw))
            xt = G.tensor(G.F32, [K, 1, 1, 1], data=_np_ptr(x))
            node = G.mul_mat_node(w, xt, _np_ptr(y), N)
            for _ in range(20):
                y[:] = 0
                if not be.compute([node]):
                    errors.append("compute failed")
                    return
                s = np.abs(y - expected[tid]).max()
                if s > 1e-3 * max(1.0, np.abs(expected[tid]).max()):
                    errors.append(f"thread {tid}: maxabs {s}")

        th = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
        [x.start() for x in th]
        [x.join() for x in th]
    assert not errors, errors[:4]


def test_mma_split_shapes_interleaved_and_deterministic(cuda, G, O):
    """The MMA path splits K into slices and tiles across warps (unit mode)
    or whole tiles across CTAs (tile mode), with per-tile arrival counters
    that every launch must find cleared: shapes that share one stream's
    scratch, interleaved, give the oracle's result each time and identical
    bits on repeats (fixed summation order)."""
    cases = [(G.Q4_K, 2048, 256 * 43), (G.Q4_0, 1024, 5120), (G.Q4_K, 64, 512), (G.Q4_K, 4096, 256 * 42),
             (G.Q4_0, 16, 256), (G.Q4_K, 16384, 2048)]
    data = []
    for i, (t, N, K) in enumerate(cases):
        raw = O.quantize(t, normal_weights(N, K, seed=900 + i))
        x = normal_x(K, seed=950 + i)
        data.append((t, N, K, raw, x, O.gemv(t, raw, N, K, x)))
    first = {}
    for rep in range(2):
        for i, (t, N, K, raw, x, ref) in enumerate(data):
            y = gemv_gpu(cuda, G, t, raw, N, K, x)
            check_parity(y, ref, f"{G.TYPE_NAME[t]} {N}x{K} rep {rep}")
            if rep == 0:
                first[i] = y
            else:
                np.testing.assert_array_equal(y, first[i])


def test_compute_graph_fuses_nodes_sharing_x(cuda, G, O):
    """q / k / v (and gate / up) style nodes: consecutive MUL_MATs on one
    device-resident x with resident MMA-layout weights run as one fused
    launch; each output matches the oracle, and so does a node that consumes
    a fused output (it must not be fused with its producers)."""
    K = 2048
    shapes = [(2048, G.Q4_K), (256, G.Q4_K), (256, G.Q4_K), (512, G.Q4_K)]  # q, k, v, then o reads q
    raws = [O.quantize(t, normal_weights(N, K, seed=60 + i)) for i, (N, t) in enumerate(shapes)]
    x = normal_x(K, seed=61)
    with G.Backend(0) as be:
        buf = G.Buffer(sum(r.nbytes for r in raws) + 8 * 8192, dev=0)
        ws = []
        for (N, t), raw in zip(shapes, raws):
            w = buf.alloc(G.tensor(t, [K, N, 1, 1]))
            buf.set(w, _np_ptr(raw), 0, raw.nbytes)
            ws.append(w)
        d_x = to_dev(cuda, x)
        ys = [cuda.full((N,), float("nan"), dtype=cuda.float32, device="cuda") for N, _ in shapes]
        xt = G.tensor(G.F32, [K, 1, 1, 1], data=d_x.data_ptr())
        qt = G.tensor(G.F32, [K, 1, 1, 1], data=ys[0].data_ptr())  # o's input: q's output (N_q == K)
        nodes = [G.mul_mat_node(ws[i], xt, ys[i].data_ptr(), shapes[i][0], name=f"n{i}") for i in range(3)]
        nodes.append(G.mul_mat_node(ws[3], qt, ys[3].data_ptr(), shapes[3][0], name="o"))
        for rep in range(2):
            assert be.compute(nodes), G.last_error()
            be.synchronize()
            got = [y.cpu().numpy() for y in ys]
            for i in range(3):
                check_parity(got[i], O.gemv(shapes[i][1], raws[i], shapes[i][0], K, x), f"fused node {i} rep {rep}")
            check_parity(got[3], O.gemv(G.Q4_K, raws[3], shapes[3][0], K, got[0]), f"consumer rep {rep}")
        buf.free()


# A decode-style chain of MMA launches, each reading an output of the one
# before: (output, type, N, input).  K of a node = N of its input; "h0" is the
# chain's input (K = 1024).  a0/a1/a2 and c0/c1 share x (fused launches); the
# Q6_K and Q3_K consumers take 16-value x blocks.
CHAIN = [("a0", "Q4_K", 1024, "h0"), ("a1", "Q4_K", 256, "h0"), ("a2", "Q4_K", 256, "h0"),
         ("b", "IQ4_XS", 512, "a0"), ("c0", "Q5_K", 768, "b"), ("c1", "Q5_K", 768, "b"),
         ("d", "Q6_K", 512, "c0"), ("e", "Q3_K", 256, "d"), ("f", "Q4_0", 512, "e")]


def run_chain(cuda, G, O, one_call: bool):
    """Runs CHAIN through compute_graph (one call for the whole chain, or one
    call per node, where no launch can prepare the next one's x) and returns
    the raw weights and the outputs of every node."""
    dims = {"h0": 1024}
    for out, _, N, _ in CHAIN:
        dims[out] = N
    raws = {out: O.quantize(G.CLAIMED[t], normal_weights(N, dims[src], seed=300 + i), nthreads=4)
            for i, (out, t, N, src) in enumerate(CHAIN)}
    with G.Backend(0) as be:
        buf = G.Buffer(sum(r.nbytes for r in raws.values()) + 16 * 8192, dev=0)
        acts = {"h0": to_dev(cuda, normal_x(1024, seed=299))}
        for out, _, N, _ in CHAIN:
            acts[out] = cuda.full((N,), float("nan"), dtype=cuda.float32, device="cuda")
        nodes = []
        for out, t, N, src in CHAIN:
            w = buf.alloc(G.tensor(G.CLAIMED[t], [dims[src], N, 1, 1]))
            buf.set(w, _np_ptr(raws[out]), 0, raws[out].nbytes)
            xt = G.tensor(G.F32, [dims[src], 1, 1, 1], data=acts[src].data_ptr())
            nodes.append(G.mul_mat_node(w, xt, acts[out].data_ptr(), N, name=out))
        if one_call:
            assert be.compute(nodes), G.last_error()
        else:
            for n in nodes:
                assert be.compute([n]), G.last_error()
        be.synchronize()
        got = {k: v.cpu().numpy() for k, v in acts.items()}
        buf.free()
    return raws, got


def test_compute_graph_chain_prepares_next_x(cuda, G, O):
    """Within one compute_graph call a launch whose output is the next
    launch's x prepares that x in its epilogue (no x-preparation kernel): the
    results are bit-identical to one call per node, and every node matches the
    oracle on its actual input."""
    raws, chained = run_chain(cuda, G, O, one_call=True)
    _, single = run_chain(cuda, G, O, one_call=False)
    for out, t, N, src in CHAIN:
        np.testing.assert_array_equal(chained[out], single[out], err_msg=out)
        check_parity(chained[out], O.gemv(G.CLAIMED[t], raws[out], N, chained[src].size, chained[src]), out)


def test_compute_graph_chain_trace_shows_prepared_x(cuda):
    """The node trace (XDNA_TRACE_NODES) of the chain: every launch after the
    first reads an x prepared by the launch before it."""
    import subprocess
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    code = ("import sys; sys.path[:0] = [%r, %r, %r]; import torch, ggml_b200 as G, oracle as O; "
            "import test_gemv_gpu as T; T.run_chain(torch, G, O, True)"
            % (here, os.path.join(here, "..", "xdna.cpp_b200"), os.path.join(here, "..", "oracle")))
    env = dict(os.environ, XDNA_TRACE_NODES="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stderr.splitlines() if "[b200 trace]" in ln]
    assert len(lines) == len(CHAIN), r.stderr[-2000:]
    ready = [ln for ln in lines if "x from the previous launch" in ln]
    # launches: (a0 a1 a2) b (c0 c1) d e f -> 6, all but the first read a prepared x
    assert len(ready) == 1 + 2 + 1 + 1 + 1, "\n".join(lines)


@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "Q4_0"])
def test_compute_graph_m_rows_with_resident_weights(cuda, G, O, name):
    """M > 1 (prefill rows) is claimed for weights resident in a B200 buffer,
    as the reference's ggml path claims it for its own buffers
    (src/ggml-xdna.cpp:81-93, 109-111); each row of the output matches the
    oracle.  Host-resident weights stay M == 1 only."""
    t = G.CLAIMED[name]
    N, K, M = 256, 1024, 3
    raw = O.quantize(t, normal_weights(N, K, seed=70))
    X = np.stack([normal_x(K, seed=71 + m) for m in range(M)]).astype(np.float32)
    with G.Backend(0) as be:
        host_w = G.tensor(t, [K, N, 1, 1], data=_np_ptr(raw))
        xt_h = G.tensor(G.F32, [K, M, 1, 1], data=_np_ptr(X))
        assert not be.supports_op(G.mul_mat_node(host_w, xt_h, None, N, M))
        buf = G.Buffer(raw.nbytes + 8192, dev=0)
        w = buf.alloc(G.tensor(t, [K, N, 1, 1]))
        buf.set(w, _np_ptr(raw), 0, raw.nbytes)
        d_x = to_dev(cuda, X)
        d_y = cuda.full((M, N), float("nan"), dtype=cuda.float32, device="cuda")
        xt = G.tensor(G.F32, [K, M, 1, 1], data=d_x.data_ptr())
        node = G.mul_mat_node(w, xt, d_y.data_ptr(), N, M)
        assert be.supports_op(node)
        assert be.compute([node]), G.last_error()
        Y = d_y.cpu().numpy()
        for m in range(M):
            check_parity(Y[m], O.gemv(t, raw, N, K, X[m]), f"{name} row {m}")
        buf.free()


@pytest.mark.parametrize("name,N,K", [("Q4_0", 512, 256), ("Q4_K", 512, 1024), ("Q6_K", 256, 2048),
                                      ("IQ3_S", 96, 512)])
def test_gemv_bf16_entry(cuda, G, O, name, N, K):
    """b200_gemv_bf16 = reference run_bf16 / run_quant_bf16 (src/xdna-gemv-engine.cpp:
    1894-1908, 1994-2009): exact BF16 -> F32, then the same GEMV."""
    t = G.CLAIMED[name]
    raw = O.quantize(t, normal_weights(N, K, seed=404 + K))
    xb = O.f32_to_bf16(normal_x(K, seed=405))
    x = (xb.astype(np.uint32) << 16).view(np.float32)
    stream = cuda.cuda.current_stream().cuda_stream
    d_raw = to_dev(cuda, raw)
    d_pk = cuda.empty_like(d_raw)
    d_xb = to_dev(cuda, xb)
    d_y = cuda.full((N,), float("nan"), dtype=cuda.float32, device="cuda")
    L = G.lib()
    G.check(L.b200_repack(t, d_raw.data_ptr(), d_pk.data_ptr(), N, K, stream), "repack")
    G.check(L.b200_gemv_bf16(t, d_pk.data_ptr(), d_xb.data_ptr(), d_y.data_ptr(), N, K, stream, 0), "gemv_bf16")
    cuda.cuda.synchronize()
    ref = O.gemv_q4_0_bf16(raw, N, K, xb) if t == G.Q4_0 else O.gemv(t, raw, N, K, x)
    check_parity(d_y.cpu().numpy(), ref, f"{name} bf16")


def test_compute_graph_replays_repeated_device_lists(cuda, G, O):
    """A node list seen again (all operands on the device) is captured into a
    CUDA graph on its second call and replayed after that: new x contents at
    the same addresses must give new, correct outputs, and a changed list
    must run correctly too (eagerly, then captured again)."""
    K = 1024
    shapes = [(512, G.Q4_K), (256, G.Q6_K), (96, G.IQ4_XS)]  # MMA, MMA, stripe layout
    raws = [O.quantize(t, normal_weights(N, K, seed=80 + i)) for i, (N, t) in enumerate(shapes)]
    with G.Backend(0) as be:
        buf = G.Buffer(sum(r.nbytes for r in raws) + 8 * 8192, dev=0)
        ws = []
        for (N, t), raw in zip(shapes, raws):
            w = buf.alloc(G.tensor(t, [K, N, 1, 1]))
            buf.set(w, _np_ptr(raw), 0, raw.nbytes)
            ws.append(w)
        d_x = cuda.empty(K, dtype=cuda.float32, device="cuda")
        ys = [cuda.empty(N, dtype=cuda.float32, device="cuda") for N, _ in shapes]
        xt = G.tensor(G.F32, [K, 1, 1, 1], data=d_x.data_ptr())
        nodes = [G.mul_mat_node(ws[i], xt, ys[i].data_ptr(), shapes[i][0], name=f"g{i}") for i in range(3)]
        for call in range(4):
            x = normal_x(K, seed=90 + call)
            d_x.copy_(cuda.from_numpy(x))
            lst = nodes if call < 3 else nodes[:2]  # the fourth call changes the list
            assert be.compute(lst), G.last_error()
            be.synchronize()
            for i in range(len(lst)):
                check_parity(ys[i].cpu().numpy(), O.gemv(shapes[i][1], raws[i], shapes[i][0], K, x), f"call {call} node {i}")
        buf.free()


def test_compute_graph_pinned_host_input_and_output(cuda, G, O):
    """A chain whose first input and last output sit in page-locked host
    memory (a decode step's token vector and logits): compute_graph runs it on
    device copies of those two operands, so the list is fused, chained and,
    from its second call, replayed as a CUDA graph.  Three calls with a new
    input in the same host buffer (eager, captured, replayed); every node
    against the oracle on its actual input each time, and the host output
    equal to the device-side result."""
    torch = cuda
    chain = [("a0", "Q4_K", 1024, "h0"), ("a1", "Q4_K", 512, "h0"), ("b", "Q4_K", 768, "a0"),
             ("c", "Q6_K", 512, "b")]
    dims = {"h0": 2048}
    for out, _, N, _ in chain:
        dims[out] = N
    raws = {out: O.quantize(G.CLAIMED[t], normal_weights(N, dims[src], seed=1300 + i), nthreads=4)
            for i, (out, t, N, src) in enumerate(chain)}
    h_host = torch.empty(dims["h0"], dtype=torch.float32, pin_memory=True)
    out_host = torch.empty(dims["c"], dtype=torch.float32, pin_memory=True)
    with G.Backend(0) as be:
        buf = G.Buffer(sum(r.nbytes for r in raws.values()) + 16 * 8192, dev=0)
        acts = {k: torch.zeros(n, dtype=torch.float32, device="cuda") for k, n in dims.items() if k not in ("h0", "c")}
        nodes = []
        for out, t, N, src in chain:
            w = buf.alloc(G.tensor(G.CLAIMED[t], [dims[src], N, 1, 1]))
            buf.set(w, _np_ptr(raws[out]), 0, raws[out].nbytes)
            xp = h_host.data_ptr() if src == "h0" else acts[src].data_ptr()
            yp = out_host.data_ptr() if out == "c" else acts[out].data_ptr()
            xt = G.tensor(G.F32, [dims[src], 1, 1, 1], data=xp)
            nodes.append(G.mul_mat_node(w, xt, yp, N, name=out))
        for call in range(3):
            h = normal_x(dims["h0"], seed=1400 + call)
            h_host.copy_(torch.from_numpy(h))
            assert be.compute(nodes), G.last_error()
            be.synchronize()
            got = {k: v.cpu().numpy() for k, v in acts.items()}
            got["h0"], got["c"] = h, out_host.numpy().copy()
            for out, t, N, src in chain:
                check_parity(got[out], O.gemv(G.CLAIMED[t], raws[out], N, dims[src], got[src]), f"call {call} {out}")
        buf.free()
