import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


@pytest.fixture(scope="session")
def cuda_device():
    """Fails loudly (not skips) when a GPU test runs without a usable device."""
    import torch
    assert torch.cuda.is_available(), "GPU test collected on a machine without CUDA"
    from hypno_b200 import build
    build.build()
    return torch.device("cuda:0")
