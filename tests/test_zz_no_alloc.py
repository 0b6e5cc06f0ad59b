"""b200_gemv_noalloc: the GEMV entry point that allocates no device memory.

It must give what b200_gemv gives (same kernels; the MMA path with its
scratch in a fixed static device array), on consecutive calls, whether this
file runs alone or after the rest of the suite, and reject shapes whose
scratch would not fit the array.  Collected last on purpose (file name).
"""
import numpy as np
import pytest

from helpers import check_parity, normal_weights, normal_x, to_dev

pytestmark = pytest.mark.gpu

# (type, N, K): every format takes the MMA path (scratch in the static array)
# when N % 16 == 0 and K % 256 == 0: Q4_K and Q4_0 (32-value x blocks), a
# tall Q4_K matrix, Q6_K (16-value x blocks) and IQ2_S (grid decode, 16-value
# x blocks).  N % 16 != 0 takes the stripe layout, which needs no scratch
# (Q4_K with N = 4104).
CASES = [("Q4_K", 4096, 4096), ("Q4_0", 2048, 5120), ("Q4_K", 16384, 2048), ("Q6_K", 256, 1024),
         ("IQ2_S", 4096, 4096), ("Q4_K", 4104, 2048)]


@pytest.mark.parametrize("name,N,K", CASES)
def test_noalloc_matches_gemv_on_consecutive_calls(cuda, G, O, name, N, K):
    torch = cuda
    t = G.CLAIMED[name]
    L = G.lib()
    raw = O.quantize(t, normal_weights(N, K, seed=4242 + N))
    x = normal_x(K, seed=77 + K)
    stream = torch.cuda.current_stream().cuda_stream
    d_raw = to_dev(torch, raw)
    d_pk = torch.empty_like(d_raw)
    d_x = to_dev(torch, x)
    y_ref = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    G.check(L.b200_repack(t, d_raw.data_ptr(), d_pk.data_ptr(), N, K, stream), "repack")
    G.check(L.b200_gemv(t, d_pk.data_ptr(), d_x.data_ptr(), y_ref.data_ptr(), N, K, stream, 0), "gemv")
    ys = [torch.full((N,), float("nan"), dtype=torch.float32, device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for y in ys:  # two calls in a row on one stream
        G.check(L.b200_gemv_noalloc(t, d_pk.data_ptr(), d_x.data_ptr(), y.data_ptr(), N, K, stream), "noalloc")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before, "b200_gemv_noalloc changed free device memory"
    ref = y_ref.cpu().numpy()
    oracle = O.gemv(t, raw, N, K, x)
    for i, y in enumerate(ys):
        got = y.cpu().numpy()
        check_parity(got, ref, f"{name} {N}x{K} call {i} vs b200_gemv")
        check_parity(got, oracle, f"{name} {N}x{K} call {i} vs oracle")


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda, G):
    torch = cuda
    L = G.lib()
    N, K = 16, 256 * 1024  # 2 MiB of x digits alone: more than the fixed area
    w = torch.zeros(16, dtype=torch.uint8, device="cuda")  # never read: rejected before any launch
    x = torch.zeros(K, dtype=torch.float32, device="cuda")
    y = torch.zeros(N, dtype=torch.float32, device="cuda")
    rc = L.b200_gemv_noalloc(G.Q4_K, w.data_ptr(), x.data_ptr(), y.data_ptr(), N, K,
                             torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    msg = G.last_error()
    assert "b200_gemv_noalloc" in msg and "fixed" in msg and "bytes" in msg, msg
    torch.cuda.synchronize()
