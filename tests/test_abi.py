"""The C ABI boundary on the CPU: the library loads without a GPU, exports every
function include/dgxm_sp.h declares, the ctypes bindings cover exactly those
functions, and every ctypes struct has the C struct's size and field offsets
(measured by compiling the header with gcc)."""
from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "dgxm_sp.h"

# ctypes class -> C struct name
STRUCTS = {
    "AttnDesc": "dgxm_attn_desc",
    "AttnExtras": "dgxm_attn_extras",
    "AttnRoute": "dgxm_attn_route",
    "A2ADesc": "dgxm_a2a_desc",
    "PrologueDesc": "dgxm_prologue_desc",
    "SeqGatherDesc": "dgxm_seq_gather_desc",
    "QkvGemmDesc": "dgxm_qkv_gemm_desc",
    "QkvStream": "dgxm_qkv_stream",
    "QuantItem": "dgxm_quant_item",
}


def header_functions() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"^[A-Za-z_][\w \t\*]*?\b(dgxm_\w+)\s*\(", text, flags=re.M))


@pytest.fixture(scope="module")
def library():
    from dgx_monarch_b200 import _build, _lib

    if not _build.LIB_PATH.exists():
        if shutil.which("nvcc") is None:
            pytest.skip("libdgxm_sp.so is not built and nvcc is absent")
        _build.build_library()
    return _lib.load()


def test_header_declares_the_entry_points():
    names = header_functions()
    for must in ("dgxm_attn_fwd", "dgxm_attn_fwd_ext", "dgxm_ulysses_scatter", "dgxm_ring_attn_fwd",
                 "dgxm_ring_attn_fwd_noalloc", "dgxm_full_context_attn_fwd", "dgxm_comm_barrier",
                 "dgxm_qkv_gemm_prologue_scatter", "dgxm_shared_amax_scale", "dgxm_seq_allgather"):
        assert must in names


def test_library_exports_every_declared_function(library):
    missing = [name for name in sorted(header_functions()) if not hasattr(library, name)]
    assert not missing, f"declared but not exported: {missing}"


def test_bindings_cover_exactly_the_declared_functions():
    from dgx_monarch_b200 import _lib

    declared = header_functions()
    bound = set(_lib.SIGNATURES)
    assert declared - bound == set(), f"declared without a ctypes binding: {sorted(declared - bound)}"
    assert bound - declared == set(), f"bound but not declared: {sorted(bound - declared)}"


def test_abi_version_without_a_gpu(library):
    assert library.dgxm_abi_version() == 2
    assert isinstance(library.dgxm_last_error_message(), bytes)


def test_invalid_arguments_fail_before_any_device_work(library):
    """A NULL descriptor is refused with DGXM_ERR_INVALID and a message, no GPU touched."""
    from dgx_monarch_b200 import _lib

    rc = library.dgxm_attn_fwd(None, None, None, None, None, None, None, None, None, None)
    assert rc == _lib.DGXM_ERR_INVALID
    assert b"descriptor" in library.dgxm_last_error_message()


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc is absent")
def test_struct_layouts_match_the_header(tmp_path):
    from dgx_monarch_b200 import _lib

    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {"]
    expected = {}
    for cls_name, c_name in STRUCTS.items():
        cls = getattr(_lib, cls_name)
        lines.append(f'  printf("{cls_name} size %zu\\n", sizeof({c_name}));')
        expected[f"{cls_name} size"] = ctypes.sizeof(cls)
        for field, _ in cls._fields_:
            lines.append(f'  printf("{cls_name}.{field} %zu\\n", offsetof({c_name}, {field}));')
            expected[f"{cls_name}.{field}"] = getattr(cls, field).offset
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    exe = tmp_path / "layout"
    src.write_text("\n".join(lines))
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    measured = {}
    for line in out.splitlines():
        key, value = line.rsplit(" ", 1)
        measured[key] = int(value)
    mismatched = {k: (v, measured.get(k)) for k, v in expected.items() if measured.get(k) != v}
    assert not mismatched, f"ctypes vs C (ctypes, C): {mismatched}"
