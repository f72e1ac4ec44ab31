"""Shared fixtures. GPU tests are marked `gpu` and need the built library and a CUDA device."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the built kernels")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tokengate_b200 import _lib
    _lib.lib()  # fail loudly if the library is missing
    return torch.device("cuda", 0)
