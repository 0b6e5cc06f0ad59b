"""GPU parity of the opt-in MMA kernels.

XDNA_B200_GEMV selects, once per process, the kernel that serves MMA-layout
launches: the default streaming kernel, or "ring" (a per-warp shared-memory
ring filled by bulk copies), "bulk" or "bulkx" (a producer warp and 16
consumer warps over a bulk-copy ring; bulkx also stages the x fragments).
Each variant runs here in a child process of its own, against the oracle at
the north_star bar, on a unit-mode and a tile-mode shape (and, for the bulk
kernels, their split and whole-tile modes).
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import os, sys
root = sys.argv[1]
for sub in ("xdna.cpp_b200", "oracle", "tests"):
    sys.path.insert(0, os.path.join(root, sub))
import torch
import ggml_b200 as G
import oracle as O
from helpers import check_parity, gemv_gpu, normal_weights, normal_x

torch.cuda.init()
# (format, N, K): unit mode (more than 64 units per SM) and tile mode; for the
# bulk kernels K = 8192 is split mode and K <= 2048 whole-tile mode
cases = [("Q4_K", 8192, 8192), ("IQ3_S", 8192, 8192), ("Q6_K", 1024, 2048), ("Q4_0", 2048, 1024)]
for i, (name, N, K) in enumerate(cases):
    t = G.CLAIMED[name]
    raw = O.quantize(t, normal_weights(N, K, seed=1700 + i), nthreads=4)
    x = normal_x(K, seed=1750 + i)
    y = gemv_gpu(torch, G, t, raw, N, K, x)
    check_parity(y, O.gemv(t, raw, N, K, x, nthreads=4), f"{os.environ['XDNA_B200_GEMV']} {name} {N}x{K}")
print("variant ok")
"""


@pytest.mark.parametrize("variant", ["ring", "bulk", "bulkx"])
def test_opt_in_kernel_matches_oracle(variant):
    env = dict(os.environ, XDNA_B200_GEMV=variant)
    r = subprocess.run([sys.executable, "-c", SCRIPT, ROOT], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "variant ok" in r.stdout, (r.stdout[-2000:], r.stderr[-2000:])
