import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device")
    config.addinivalue_line("markers", "slow: larger CPU cases")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def ref():
    from oracle import oracle as o
    if not o.ref_available():
        pytest.skip("reference sources/library not present (GPU box)")
    return o.ref(1)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from warp_b200 import ffi
    ffi.load()
    assert ffi.load().warp_device_ok(0) == 1, "device 0 is not an sm_100 part"
    return torch.device("cuda", 0)
