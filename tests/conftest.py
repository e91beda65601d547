import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: a larger case")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test is marked gpu and needs a CUDA device")
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def bits(a):
    import numpy as np

    return np.asarray(a, dtype=np.float32).view(np.uint32)
