import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "tilelang-fa-v100_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libfa_b200.so")


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "GPU tests need an sm_100 (B200-class) device"
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _no_device_error(request):
    """Every GPU test also checks the library's device error word (bounded waits)."""
    yield
    if request.node.get_closest_marker("gpu") is not None:
        import torch
        if torch.cuda.is_available():
            from tilelang_fa_v100 import _ext
            code, site, block = _ext.read_device_error(clear=True)
            assert code == 0, "device error %d at site %d (block %d)" % (code, site, block)
