"""Row sharding across ranks, on CPU: two `gloo` ranks split the rows of one
weight matrix with ggml_backend_xdna_shard_rows, each computes its slice (the
CPU oracle stands in for the GPU kernel), and an all-gather in rank order
rebuilds y.  The GPU path does the same with the kernel and NCCL; rows are
independent, so the gathered result must equal the unsharded one bit for bit.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

WORLD = 2


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank: int, port: int, t: int, N: int, K: int, out_dir: str) -> None:
    import ctypes as C
    import sys

    import torch
    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for sub in ("xdna.cpp_b200", "oracle", "tests"):
        sys.path.insert(0, os.path.join(root, sub))
    import ggml_b200 as G
    import oracle as O
    from helpers import normal_weights, normal_x

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    try:
        w = O.quantize(t, normal_weights(N, K, seed=21), nthreads=1)  # every rank builds the same matrix
        x = normal_x(K, seed=22)
        r0, nr = C.c_int64(), C.c_int64()
        assert G.lib().ggml_backend_xdna_shard_rows(N, WORLD, rank, C.byref(r0), C.byref(nr)) == 0
        rb = O.row_bytes(t, K)
        mine = w[r0.value * rb:(r0.value + nr.value) * rb]
        y_local = torch.from_numpy(O.gemv(t, mine, nr.value, K, x, nthreads=1))
        parts = [torch.empty_like(y_local) for _ in range(WORLD)]
        dist.all_gather(parts, y_local)
        if rank == 0:
            np.save(os.path.join(out_dir, "y_sharded.npy"), torch.cat(parts).numpy())
            np.save(os.path.join(out_dir, "y_full.npy"), O.gemv(t, w, N, K, x, nthreads=1))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("t,N,K", [(2, 256, 512), (12, 512, 1024), (21, 128, 512)])
def test_row_sharded_gemv_matches_unsharded(tmp_path, t, N, K):
    import torch.multiprocessing as mp

    mp.start_processes(worker, args=(free_port(), t, N, K, str(tmp_path)), nprocs=WORLD, join=True,
                       start_method="spawn")
    np.testing.assert_array_equal(np.load(tmp_path / "y_sharded.npy"), np.load(tmp_path / "y_full.npy"))
