import os
import shutil
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def autlib():
    """libautdot.so, built in-tree when missing or stale (needs nvcc)."""
    from accessor_universal_test_b200 import _lib, build
    if shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc"):
        build.build_library()
    return _lib.load()


@pytest.fixture(scope="session")
def orc():
    import pyoracle
    return pyoracle.oracle()


@pytest.fixture(scope="session")
def ref():
    """The reference's own host code, or skip when its tree is absent."""
    import pyoracle
    r = pyoracle.reference()
    if r is None:
        pytest.skip("reference tree not available on this machine")
    return r


@pytest.fixture(scope="session")
def ws(autlib):
    from accessor_universal_test_b200 import _lib
    w = _lib.Workspace(0)
    yield w
    w.close()
