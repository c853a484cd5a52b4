"""Shared pytest configuration.

``-m "not gpu"`` runs here without a GPU (oracle vs golden fixtures, host logic,
library exports); ``-m gpu`` tests need a B200 and call the CUDA path through
the C ABI.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); calls the sm_100a kernels")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
