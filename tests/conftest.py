"""Shared pytest configuration: the ``gpu`` marker and common fixtures."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def cuda():
    """Initialises the library on cuda:0 (GPU tests only)."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    from magma_b200 import ops

    torch.cuda.set_device(0)
    ops.init(0)
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.build()
    return o
