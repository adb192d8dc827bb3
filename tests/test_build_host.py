"""The in-tree build's options, on the CPU."""
from __future__ import annotations

import pytest


def test_tuning_defines_accept_only_the_kernel_macros(monkeypatch):
    from dgx_monarch_b200 import _build

    monkeypatch.setenv("DGXM_NVCC_DEFINES", "-DDGXM_SM_POLY_MOD=4 -DDGXM_SM_THR_BF16=6.0f")
    assert _build.tuning_defines() == ["-DDGXM_SM_POLY_MOD=4", "-DDGXM_SM_THR_BF16=6.0f"]
    monkeypatch.setenv("DGXM_NVCC_DEFINES", "-O0")
    with pytest.raises(ValueError, match="DGXM_"):
        _build.tuning_defines()
    monkeypatch.delenv("DGXM_NVCC_DEFINES")
    assert _build.tuning_defines() == []
