import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    return O


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    """The CUDA library on a GPU; a GPU test without a GPU is an error, not a skip."""
    import torch
    assert torch.cuda.is_available(), "gpu-marked test needs a CUDA device"
    from tcc_b200 import build
    build.build()
    from tcc_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")
