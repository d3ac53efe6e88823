import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); runs the CUDA kernels")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for GPU tests. A GPU test never skips: without a device
    it fails, so a run on a box whose CUDA is broken cannot pass silently."""
    import torch
    assert torch.cuda.is_available(), "GPU test without a CUDA device"
    torch.cuda.init()
    return torch.device("cuda:0")
