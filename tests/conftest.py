import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_PARENT = os.path.join(ROOT, "ml-edsl_b200")
for p in (ROOT, PKG_PARENT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


@pytest.fixture(scope="session")
def cuda():
    """The torch CUDA device; GPU tests fail loudly (not skip) without one."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    return torch.device("cuda:0")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Builds the native library and the oracle once per session if stale."""
    sys.path.insert(0, ROOT)
    import oracle
    oracle.build()
    from importlib import import_module
    build = import_module("build")  # ml-edsl_b200/build.py
    build.build()
