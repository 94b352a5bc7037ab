import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "fhe-ssm_b200")
for p in (ROOT, PKG_DIR, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the engine against the oracle")


_CUDA = None


def cuda_available():
    """True when the CUDA driver reports at least one device (checked through libcuda)."""
    global _CUDA
    if _CUDA is None:
        try:
            import ctypes
            cu = ctypes.CDLL("libcuda.so.1")
            n = ctypes.c_int(0)
            _CUDA = cu.cuInit(0) == 0 and cu.cuDeviceGetCount(ctypes.byref(n)) == 0 and n.value > 0
        except OSError:
            _CUDA = False
    return _CUDA


def pytest_collection_modifyitems(config, items):
    if cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
