import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for gpu-marked tests; fails (does not skip) without one."""
    import torch

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    from webyiq_b200 import _lib

    _lib.load()
    return torch.device("cuda:0")
