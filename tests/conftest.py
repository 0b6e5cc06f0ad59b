"""Test configuration: import paths and the `gpu` marker.

CPU tests (`-m "not gpu"`) cover the oracle against the reference's golden
vectors, the host-side layout logic and the C ABI surface; GPU tests
(`-m gpu`) are the parity tests proper and call the kernels through the C ABI.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("xdna.cpp_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def G():
    import ggml_b200

    ggml_b200.lib()  # fails loudly if the library is not built
    return ggml_b200


@pytest.fixture(scope="session")
def O():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device (run `-m \"not gpu\"` on CPU-only hosts)")
    torch.cuda.init()
    return torch
