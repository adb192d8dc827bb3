"""B200-native sequence-parallel attention path for dgx-monarch.

A drop-in behind the reference's USP attention seam (adapters/base.py:216-326):
hand-written sm_100a CUDA in libdgxm_sp.so, reached through a C ABI
(include/dgxm_sp.h), with the Python host side mirroring the reference's
callable contract.
"""
from __future__ import annotations

__all__ = ["ops"]
