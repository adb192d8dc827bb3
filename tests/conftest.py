from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libdgxm_sp.so")


def _has_cuda() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover - torch import problems surface elsewhere
        return False


def pytest_collection_modifyitems(config, items):
    if _has_cuda():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def lib():
    """The built C-ABI library (built on first use; no fallback)."""
    from dgx_monarch_b200 import _build, _lib

    _build.build_library()
    return _lib.load()


@pytest.fixture(autouse=True)
def _clean_device_error(request):
    """Every GPU test must leave the device error word clean."""
    yield
    if "gpu" in request.keywords and _has_cuda():
        from dgx_monarch_b200 import _lib

        assert _lib.device_error(clear=True) == 0, "a bounded device wait expired"


os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
