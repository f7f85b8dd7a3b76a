import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "mamba-3-lite_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


def cuda_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda_device():
    if not cuda_available():
        pytest.skip("no CUDA device")
    import torch
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_status_checked(request, monkeypatch):
    """GPU tests run with M3SSD_CHECK=1: every operator call synchronises and raises if a kernel's
    bounded wait expired (a hand-off that never came), so a slow-but-correct timeout cannot pass."""
    if request.node.get_closest_marker("gpu") is not None:
        monkeypatch.setenv("M3SSD_CHECK", "1")
