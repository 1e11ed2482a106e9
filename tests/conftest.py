import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA libraries")


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test: the kernels' watchdog status word must be zero
    (no bounded wait in any kernel gave up)."""
    yield
    if request.node.get_closest_marker("gpu") is None or not cuda_ok():
        return
    from blockfp8_b200 import _native
    if _native.capi_loaded():
        status = _native.device_status(reset=True)
        assert status == 0, f"a kernel reported watchdog status {status:#x}"
