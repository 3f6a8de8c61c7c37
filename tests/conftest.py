import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run with -m 'not gpu' on a CPU box)")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        pytest.fail(f"these kernels are built for sm_100a, device is sm_{major}{minor}")
    return torch.device("cuda:0")
