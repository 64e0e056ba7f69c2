"""Shared fixtures. Tests marked `gpu` need a B200; everything else runs on the CPU."""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG_NAME = "cuda-llm-inference-engine_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def b2():
    """The host-side package (the library itself is loaded lazily on first use)."""
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    return o


@pytest.fixture(scope="session")
def cuda(b2):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    b2.load_library()
    b2.device_error(clear=True)
    return torch.device("cuda:0")
