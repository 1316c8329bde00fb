"""Shared test set-up: import paths for the product binding (b2g) and the CPU oracle."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ada-tensor-core-gemm_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda():
    """torch with a CUDA device; GPU tests fail loudly (no skip) when there is none."""
    import torch

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    major, minor = torch.cuda.get_device_capability()
    assert (major, minor) == (10, 0), f"needs sm_100 (B200), got sm_{major}{minor}"
    return torch
