"""Shared pytest configuration.

Marker ``gpu``: the test needs a CUDA device with compute capability 10.0
(B200, sm_100a); the suite run without ``-m gpu`` only covers the oracle, the
golden fixtures, the host-side logic and the C-ABI library's exports.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "mps-fp8-for-torch-and-comfyui-python-package_b200")
for p in (ROOT, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


def has_sm100() -> bool:
    import torch
    if not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability(0) == (10, 0)


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def device():
    if not has_sm100():
        pytest.fail("gpu-marked test needs a B200 (sm_100a) device")
    return "cuda"
