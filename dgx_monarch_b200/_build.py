"""Build libdgxm_sp.so in-tree with nvcc for sm_100a.

The library is one translation unit (csrc/dgxm_sp.cu) linked against the
static CUDA runtime, so it loads next to any torch build without a JIT cache.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_NAME = "libdgxm_sp.so"
LIB_PATH = PKG_DIR / LIB_NAME

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc was not found; set CUDA_HOME or put nvcc on PATH")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
                  + list((PKG_DIR.parent / "include").glob("*.h")))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(src.stat().st_mtime > built for src in sources())


def tuning_defines() -> list[str]:
    """Compile-time tuning of the kernels' defaults (the DGXM_SM_* macros of
    csrc/attn_fwd.cu), from DGXM_NVCC_DEFINES, e.g. "-DDGXM_SM_POLY_MOD=4".
    Only -D definitions are taken."""
    defines = os.environ.get("DGXM_NVCC_DEFINES", "").split()
    bad = [d for d in defines if not d.startswith("-DDGXM_")]
    if bad:
        raise ValueError(f"DGXM_NVCC_DEFINES takes -DDGXM_* definitions only, got {bad}")
    return defines


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/dgxm_sp.cu into dgx_monarch_b200/libdgxm_sp.so.  A build
    with tuning defines is always redone, so the library matches them."""
    defines = tuning_defines()
    if not force and not defines and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, *defines]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-o", str(tmp), str(CSRC / "dgxm_sp.cu")]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        print(proc.stdout + proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(force=True, verbose=True))
