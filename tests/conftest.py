import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def golden():
    path = os.path.join(ROOT, "tests", "golden", "o3_golden.pt")
    return torch.load(path, map_location="cpu", weights_only=True)


@pytest.fixture(scope="session")
def emu_lib():
    """The host-emulation build of the kernels (same C ABI, host pointers)."""
    from flashcart_b200 import _native, build_ext

    if not os.path.exists(build_ext.EMU_LIB):
        build_ext.build(cuda=False, emu=True)
    return _native.bind(build_ext.EMU_LIB)


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)
