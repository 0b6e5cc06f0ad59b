"""Row-sharded GEMV over two GPUs through the C ABI.

Each of two processes drives one GPU with ggml_backend_xdna_init_sharded,
uploads its rows of every weight (ggml_backend_xdna_shard_rows) and runs one
compute_graph call: two nodes that share x (fused into one launch per rank)
and a third single node.  Both ranks must end with the full outputs, equal
to the oracle, over the peer exchange (rows stored into the peers' buffers
by the GEMV) and over the NCCL all-gather fallback.

Chain: the third node reads the first node's full (gathered) output, so the
gather kernel prepares its x; the list is computed three times (the second
call is captured as a CUDA graph, the third replays it) with identical
results each time.

Failure detection: a rank that skips a step must not hang the other; the
other's bounded wait ends and compute_graph reports the missing rows.

Needs two GPUs; skipped otherwise.  NVLS stays off (NCCL_NVLS_ENABLE=0).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
WORLD = 2


def _worker(rank: int, tmp: str, seed: int, mode: str = "run") -> None:
    import ctypes as C
    import sys
    import time

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for sub in ("xdna.cpp_b200", "oracle", "tests"):
        sys.path.insert(0, os.path.join(root, sub))
    import torch

    import ggml_b200 as G
    import oracle as O
    from helpers import normal_weights, normal_x

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    if mode == "nccl":
        os.environ["XDNA_B200_NO_P2P"] = "1"
    torch.cuda.set_device(rank)
    idf = os.path.join(tmp, "nccl_id")
    if rank == 0:
        with open(idf + ".tmp", "wb") as f:
            f.write(G.nccl_unique_id())
        os.replace(idf + ".tmp", idf)
    for _ in range(600):  # the id file appears within seconds
        if os.path.exists(idf):
            break
        time.sleep(0.1)
    nccl_id = open(idf, "rb").read()
    K = 2048
    mats = [(G.Q4_K, 1024), (G.Q4_K, 256), (G.Q4_0, 512)]  # two fused (same x), one single (Q4_0)
    chain = mode == "chain"
    if chain:
        mats[2] = (G.Q6_K, 512)  # reads node 0's output: K = 1024, 16-value x blocks
    x = normal_x(K, seed + 1)
    with G.Backend(rank, WORLD, rank, nccl_id) as be:
        buf = G.Buffer(sum(N * G.row_bytes(t, K) for t, N in mats) // WORLD + 64 * 1024, dev=rank)
        d_x = torch.from_numpy(x).cuda()
        outs, nodes, refs, keep = [], [], [], []
        raws = []
        for i, (t, N) in enumerate(mats):
            Ki = 1024 if chain and i == 2 else K
            raw = O.quantize(t, normal_weights(N, Ki, seed + 10 + i), nthreads=4)
            raws.append(raw)
            refs.append(O.gemv(t, raw, N, Ki, x, nthreads=4) if Ki == K else None)
            r0, nr = C.c_int64(), C.c_int64()
            G.check(G.lib().ggml_backend_xdna_shard_rows(N, WORLD, rank, C.byref(r0), C.byref(nr)), "shard_rows")
            rb = G.row_bytes(t, Ki)
            mine = np.ascontiguousarray(raw[r0.value * rb:(r0.value + nr.value) * rb])
            w = buf.alloc(G.tensor(t, [Ki, nr.value, 1, 1]))
            buf.set(w, mine.ctypes.data, 0, mine.nbytes)
            y = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
            src = outs[0] if Ki != K else d_x
            xt = G.tensor(G.F32, [Ki, 1, 1, 1], data=src.data_ptr())
            nodes.append(G.mul_mat_node(w, xt, y.data_ptr(), N, name=f"m{i}"))
            outs.append(y)
            keep += [w, xt, mine]
        done = os.path.join(tmp, "rank0_done")
        if mode == "skip" and rank == 1:
            # this rank leaves the step before it starts, but keeps its memory
            # (which rank 0's kernels still write to) until rank 0 is through
            ok, t_call = True, 0.0
            for _ in range(600):
                if os.path.exists(done):
                    break
                time.sleep(0.1)
        else:
            ok, t_call, prev, same = True, 0.0, None, True
            for _ in range(3 if chain else 1):  # chain: eager, captured, replayed
                t = time.perf_counter()
                ok = be.compute(nodes) and ok
                t_call = time.perf_counter() - t
                be.synchronize()
                got = [y.cpu().numpy().copy() for y in outs]
                same = same and (prev is None or all(np.array_equal(a, b) for a, b in zip(got, prev)))
                prev = got
            if rank == 0:
                open(done, "w").close()
        be.synchronize()
        res = {"ok": ok, "err": G.last_error() if not ok else "", "t_call": t_call}
        if chain:
            res["same"] = same
            refs[2] = O.gemv(mats[2][0], raws[2], mats[2][1], 1024, outs[0].cpu().numpy(), nthreads=4)
        for i, y in enumerate(outs):
            s = O.stats(y.cpu().numpy(), refs[i])
            res[f"cos{i}"], res[f"rel{i}"] = s["cos"], s["maxabs_rel"]
        buf.free()
    np.save(os.path.join(tmp, f"res{rank}.npy"), np.array([res], dtype=object), allow_pickle=True)


def _run(tmp_path, mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, str(tmp_path), 314, mode)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [np.load(tmp_path / f"res{r}.npy", allow_pickle=True)[0] for r in range(WORLD)]


@pytest.mark.parametrize("mode", ["run", "nccl", "chain"])
def test_row_sharded_nodes_over_two_gpus(cuda, tmp_path, mode):
    if cuda.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    from helpers import COS_MIN, MAXABS_REL

    for r, res in enumerate(_run(tmp_path, mode)):
        assert res["ok"], res
        assert res.get("same", True), res
        for i in range(3):
            assert res[f"cos{i}"] >= COS_MIN and res[f"rel{i}"] <= MAXABS_REL, (r, i, res)


def test_rank_missing_a_step_is_reported_not_hung(cuda, tmp_path):
    if cuda.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    res = _run(tmp_path, "skip")
    assert not res[0]["ok"] and "did not arrive" in res[0]["err"], res[0]
    assert res[0]["t_call"] < 30.0, res[0]
