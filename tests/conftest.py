"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked `gpu` need an sm_100 device and call the CUDA backend through
its C ABI; everything else runs on the CPU (oracle, host logic, ABI loading).
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); parity through the C ABI")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.load()
    return O


@pytest.fixture(scope="session")
def nb():
    import nexus_b200
    nexus_b200._lib.load()
    return nexus_b200


@pytest.fixture(scope="session")
def tiny_path(nb):
    return nb.model_path("tiny")


@pytest.fixture(scope="session")
def backend(nb):
    if not nb._lib.load().nexus_cuda_is_available():
        pytest.fail("no sm_100 CUDA device: the gpu tests need a B200 (the backend has no CPU fallback)")
    b = nb.CudaBackend(device=0)
    yield b
    b.close()


def seeded(seed):
    return np.random.default_rng(seed)
