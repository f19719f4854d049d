"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200) and call the sm_100a kernels
through the C ABI; everything else runs on the CPU. Tests never read the
reference checkout: golden vectors are committed under tests/golden/.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built kernel library")
    config.addinivalue_line("markers", "slow: long-running case")
    config.addinivalue_line("markers", "expects_device_timeout: the test provokes a bounded-wait timeout")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


@pytest.fixture(scope="session")
def dev():
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test, fail if any bounded device wait timed out (a
    pipeline that deadlocked would otherwise only show as wrong numbers)."""
    yield
    if "gpu" not in request.keywords or request.node.get_closest_marker("expects_device_timeout"):
        return
    import torch
    if not torch.cuda.is_available():
        return
    from neso_b200 import _lib
    rc = _lib.lib().neso_device_status(0, None, None, None, None)
    if rc != _lib.NESO_OK:
        msg = _lib.last_error()
        _lib.lib().neso_clear_device_status(0)
        pytest.fail(f"device status after test: {msg}")
