import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: long CPU test")


import pytest  # noqa: E402


@pytest.fixture(autouse=True)
def _no_device_error_words(request):
    """After every GPU test, no kernel may have recorded a device-side error word (timeouts of
    bounded waits, plan mismatches, skipped out-of-range accesses)."""
    yield
    if request.node.get_closest_marker("gpu") is None or "plan_mismatch" in request.node.name:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from xsake_b200 import _lib
    code = _lib.device_error(torch.cuda.current_stream().cuda_stream)
    assert code == 0, f"device error word 0x{code:08x} recorded during {request.node.name}"
