import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs the sm_100a engine)")
    config.addinivalue_line("markers", "slow: long-running (large synthetic models)")


def _cuda_available() -> bool:
    try:
        import ctypes
        rt = ctypes.CDLL("libcuda.so.1")
        n = ctypes.c_int(0)
        return rt.cuInit(0) == 0 and rt.cuDeviceGetCount(ctypes.byref(n)) == 0 and n.value > 0
    except OSError:
        return False


HAVE_GPU = _cuda_available()


def pytest_collection_modifyitems(config, items):
    if HAVE_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Make sure the native libraries exist (build() is idempotent)."""
    import __graft_entry__
    __graft_entry__.build()
