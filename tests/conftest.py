import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA torch module; GPU tests fail (not skip) when CUDA is unusable."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a usable CUDA device"
    major, minor = torch.cuda.get_device_capability()
    assert (major, minor) == (10, 0), "expected a B200 (sm_100), got sm_%d%d" % (major, minor)
    return torch


@pytest.fixture(scope="session")
def tl():
    """The ternocl_b200 package with its native library loaded (raises if absent)."""
    import ternocl_b200
    ternocl_b200.lib()
    return ternocl_b200
