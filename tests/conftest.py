import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

os.environ.setdefault("VRM_TEST_MODE", "1")
os.environ.setdefault("VRM_API_TOKEN", "testtoken")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


def _has_cuda():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_cuda():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture
def cuda_errors_clean():
    """Asserts that no bounded device wait timed out during the test."""
    yield
    from vramancer_b200 import ops
    assert ops.read_and_clear_errors() == 0
