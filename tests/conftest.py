import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (runs on the B200 box)")


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def native():
    from rustgears_b200 import _native
    return _native


@pytest.fixture(scope="session")
def gpu():
    """Skips nothing: a GPU test that finds no device fails loudly."""
    import torch
    assert torch.cuda.is_available(), "gpu-marked test needs a CUDA device"
    from rustgears_b200 import _native
    assert _native.lib().rg_device_count() > 0, "no sm_100 device visible to librg_npu"
    return torch
