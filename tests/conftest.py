"""pytest configuration: the `gpu` marker, import paths and shared fixtures.

Tests marked `gpu` need a CUDA device and the built libgs3d_b200.so; everything else runs
on the CPU (the oracle, the host logic, the C ABI's exports and gloo process groups).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "custom-3dgs-cuda_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built extension")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA GPU required")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def crc(cuda_device):
    import custom_rasterizer_cuda

    return custom_rasterizer_cuda


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.build()
    return O
