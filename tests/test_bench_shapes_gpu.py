"""GPU parity at the shapes the benchmarks run, through the C ABI.

The MMA GEMV picks its work split per launch: large launches (more than 64
(tile, group) units per SM) run in unit mode, small ones in tile mode.  Every
launch of the 70B-shaped decode step is a unit-mode launch, so these cases
check unit mode for all nine formats at the step's matrix shapes, the
configs[0]/[1] Q4_0 shapes with quantised N(0, 0.02) weights, a unit-mode
prepared-x chain through compute_graph (one call, then captured and replayed),
and the reference's ne2 / ne3 loop (src/ggml-xdna.cpp:261-298) on a 4-D node.
Each output is compared with the CPU oracle at the north_star bar.
"""
import ctypes as C

import numpy as np
import pytest

from helpers import check_parity, gemv_gpu, normal_x

pytestmark = pytest.mark.gpu

TYPES = ["Q4_0", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ3_XXS", "IQ3_S", "IQ2_S", "IQ4_XS"]
SMS = 148  # B200


def quantized_normal(O, t: int, N: int, K: int, seed: int, rows_per_chunk: int = 4096) -> np.ndarray:
    """N(0, 0.02) weights quantised by the oracle, generated in row chunks so
    that the F32 matrix of a large shape never sits in host memory whole."""
    rng = np.random.default_rng(seed)
    parts = []
    for r0 in range(0, N, rows_per_chunk):
        n = min(rows_per_chunk, N - r0)
        parts.append(O.quantize(t, rng.normal(0.0, 0.02, size=(n, K)).astype(np.float32)))
    return np.concatenate(parts)


def units(N: int, K: int) -> int:
    return (N // 16) * (K // 256)


@pytest.mark.parametrize("name", TYPES)
@pytest.mark.parametrize("N,K", [(28672, 8192), (8192, 28672)])
def test_unit_mode_all_formats_at_decode_shapes(cuda, G, O, name, N, K):
    """gate/up (28672 x 8192) and down (8192 x 28672) of the 70B-shaped step."""
    assert units(N, K) > 64 * SMS  # unit mode
    t = G.CLAIMED[name]
    raw = quantized_normal(O, t, N, K, seed=5000 + N + t)
    x = normal_x(K, seed=5100 + K)
    y = gemv_gpu(cuda, G, t, raw, N, K, x)
    check_parity(y, O.gemv(t, raw, N, K, x), f"{name} {N}x{K} (unit mode)")


def test_unit_mode_lm_head_q4_k(cuda, G, O):
    """The 70B-shaped lm_head, 128256 x 8192 Q4_K (591 MB of weights)."""
    N, K = 128256, 8192
    raw = quantized_normal(O, G.Q4_K, N, K, seed=5200)
    x = normal_x(K, seed=5201)
    y = gemv_gpu(cuda, G, G.Q4_K, raw, N, K, x)
    check_parity(y, O.gemv(G.Q4_K, raw, N, K, x), "Q4_K lm_head")


@pytest.mark.parametrize("N,K", [(4096, 4096), (8192, 8192), (17408, 5120)])
def test_q4_0_configs_quantized_normal(cuda, G, O, N, K):
    """W ~ N(0, 0.02) quantised to Q4_0
    (ggml quantize_row_q4_0_ref, restated in the oracle), x ~ N(0, 1)."""
    raw = quantized_normal(O, G.Q4_0, N, K, seed=5300 + N)
    x = normal_x(K, seed=5301 + K)
    y = gemv_gpu(cuda, G, G.Q4_0, raw, N, K, x)
    check_parity(y, O.gemv(G.Q4_0, raw, N, K, x), f"Q4_0 {N}x{K}")


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# One 70B-shaped layer (Q4_K) as the bench runs it: q/k/v read h (one fused
# launch), o reads q, gate/up read o (one fused launch), down reads gate and
# writes the next h.  (output, N, input)
LAYER = [("q", 8192, "h"), ("k", 1024, "h"), ("v", 1024, "h"), ("o", 8192, "q"),
         ("gate", 28672, "o"), ("up", 28672, "o"), ("down", 8192, "gate")]


def test_unit_mode_chain_one_call_and_replay(cuda, G, O):
    """The decode step's launch plan at full size: four unit-mode launches,
    each preparing the next one's x in its epilogue.  Called three times with
    new x at the same address: the first call runs eagerly, the second is
    captured into a CUDA graph, the third replays it.  Every node matches the
    oracle on its actual input each time."""
    torch = cuda
    dims = {"h": 8192}
    for out, N, _ in LAYER:
        dims[out] = N
    raws = {out: quantized_normal(O, G.Q4_K, N, dims[src], seed=5400 + i)
            for i, (out, N, src) in enumerate(LAYER)}
    with G.Backend(0) as be:
        buf = G.Buffer(sum(r.nbytes for r in raws.values()) + 16 * 8192, dev=0)
        acts = {name: torch.zeros(n, dtype=torch.float32, device="cuda") for name, n in dims.items()}
        h_next = torch.zeros(8192, dtype=torch.float32, device="cuda")
        nodes = []
        for out, N, src in LAYER:
            w = buf.alloc(G.tensor(G.Q4_K, [dims[src], N, 1, 1]))
            buf.set(w, _ptr(raws[out]), 0, raws[out].nbytes)
            xt = G.tensor(G.F32, [dims[src], 1, 1, 1], data=acts[src].data_ptr())
            y = h_next if out == "down" else acts[out]
            nodes.append(G.mul_mat_node(w, xt, y.data_ptr(), N, name=out))
        for call in range(3):
            acts["h"].copy_(torch.from_numpy(normal_x(8192, seed=5500 + call)))
            assert be.compute(nodes), G.last_error()
            be.synchronize()
            got = {k: v.cpu().numpy() for k, v in acts.items()}
            got["down"] = h_next.cpu().numpy()
            for out, N, src in LAYER:
                check_parity(got[out], O.gemv(G.Q4_K, raws[out], N, dims[src], got[src]), f"call {call} {out}")
        buf.free()


@pytest.mark.parametrize("resident", [False, True])
def test_ne2_ne3_loop(cuda, G, O, resident):
    """A node with ne2 = 2, ne3 = 2 (reference process_mul_mat_node,
    src/ggml-xdna.cpp:261-298): four weight matrices one after the other, four
    activation rows, four output rows; and the same node with src1 broadcast
    (src1 ne2 = ne3 = 1, stride 0)."""
    t, N, K = G.Q4_K, 256, 1024
    rb = G.row_bytes(t, K)
    mats = [quantized_normal(O, t, N, K, seed=5600 + i) for i in range(4)]
    raw = np.concatenate(mats)
    X = np.stack([normal_x(K, seed=5700 + i) for i in range(4)]).astype(np.float32)
    torch = cuda
    with G.Backend(0) as be:
        buf = None
        if resident:
            buf = G.Buffer(raw.nbytes + 8192, dev=0)
            w = buf.alloc(G.tensor(t, [K, N, 2, 2]))
            buf.set(w, _ptr(raw), 0, raw.nbytes)
        else:
            w = G.tensor(t, [K, N, 2, 2], data=_ptr(raw))
        w.nb[1], w.nb[2], w.nb[3] = rb, rb * N, rb * N * 2
        for broadcast in (False, True):
            xs = X[:1] if broadcast else X
            d_x = torch.from_numpy(np.ascontiguousarray(xs)).cuda()
            d_y = torch.full((4, N), float("nan"), dtype=torch.float32, device="cuda")
            xt = G.tensor(G.F32, [K, 1, 1 if broadcast else 2, 1 if broadcast else 2], data=d_x.data_ptr())
            node = G.tensor(G.F32, [N, 1, 2, 2], data=d_y.data_ptr(), op=G.GGML_OP_MUL_MAT, name="mm4d")
            node.src[0] = C.pointer(w)
            node.src[1] = C.pointer(xt)
            assert be.supports_op(node)
            assert be.compute([node]), G.last_error()
            be.synchronize()
            Y = d_y.cpu().numpy()
            for i in range(4):
                x = X[0] if broadcast else X[i]
                check_parity(Y[i], O.gemv(t, mats[i], N, K, x), f"slice {i} broadcast={broadcast}")
        if buf is not None:
            buf.free()


@pytest.mark.parametrize("name,N,K", [("Q4_K", 256, 8192), ("Q4_K", 40, 1024), ("IQ2_S", 256, 4096),
                                      ("Q4_0", 512, 4096)])
@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_nonfinite_activations_propagate(cuda, G, O, name, N, K, bad):
    """An infinity or a NaN in x reaches every output row as a non-finite
    value, as in the reference's F32 dot products (the integer path carries
    it through the block scale); the other blocks' values do not hide it."""
    t = G.CLAIMED[name]
    raw = O.quantize(t, np.random.default_rng(5800).normal(0.0, 0.02, size=(N, K)).astype(np.float32))
    x = normal_x(K, seed=5801)
    x[K // 2 + 3] = bad
    y = gemv_gpu(cuda, G, t, raw, N, K, x)
    ref = O.gemv(t, raw, N, K, x)
    assert not np.isfinite(ref).any()
    assert not np.isfinite(y).any(), np.flatnonzero(np.isfinite(y))[:8]
