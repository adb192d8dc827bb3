"""The C ABI's error contract without a GPU: every entry point returns a
status and a message for a request it cannot run, and an empty request
succeeds as a no-op.  Each case below is refused (or is empty) by argument
checks that run before any CUDA call -- the pointers passed are aligned
placeholders that are never dereferenced -- so these tests launch nothing on
any machine."""
from __future__ import annotations

import ctypes
import shutil

import pytest

FAKE = 1 << 20  # 16-byte aligned placeholder address, never dereferenced


@pytest.fixture(scope="module")
def lib():
    from dgx_monarch_b200 import _build, _lib

    if not _build.LIB_PATH.exists():
        if shutil.which("nvcc") is None:
            pytest.skip("libdgxm_sp.so is not built and nvcc is absent")
        _build.build_library()
    return _lib.load()


def _desc(**kw):
    from dgx_monarch_b200 import _lib

    d = _lib.AttnDesc()
    d.batch, d.q_len, d.kv_len, d.q_heads, d.kv_heads, d.head_dim = 1, 16, 16, 2, 2, 128
    d.in_dtype = d.out_dtype = _lib.DTYPE_BF16
    for key, value in kw.items():
        setattr(d, key, value)
    return d


def _status(lib, rc, code, needle):
    from dgx_monarch_b200 import _lib

    assert rc == code, (rc, lib.dgxm_last_error_message())
    if code != _lib.DGXM_OK:
        assert needle in lib.dgxm_last_error_message().decode()


@pytest.mark.parametrize("kw,code,needle", [
    ({"head_dim": 96}, 2, "head_dim 96"),
    ({"head_dim": 64, "in_dtype": 2}, 2, "head_dim 64"),   # e4m3 runs 128 only
    ({"q_heads": 3}, 1, "divisible"),
    ({"kv_len": 0}, 1, "empty key axis"),
    ({"q_len": -1}, 1, "negative"),
    ({"in_dtype": 3}, 2, "input dtype"),
    ({"in_dtype": 1}, 2, "output dtype 0 is not supported for input dtype 1"),
    ({"in_dtype": 2, "out_dtype": 1}, 2, "output dtype 1"),
    ({"q_len": 0}, 0, ""),
    ({"batch": 0}, 0, ""),
])
def test_attention_argument_checks(lib, kw, code, needle):
    d = _desc(**kw)
    rc = lib.dgxm_attn_fwd(ctypes.byref(d), FAKE, FAKE, FAKE, None, None, None, FAKE, None, None)
    _status(lib, rc, code, needle)


def test_routed_attention_checks_the_route_first(lib):
    d = _desc()
    peers = (ctypes.c_void_p * 2)(FAKE, FAKE)
    rc = lib.dgxm_attn_fwd_routed(ctypes.byref(d), FAKE, FAKE, FAKE, None, None, None, None, 2, 0, 8,
                                  0, None, None)
    _status(lib, rc, 1, "o_peers")
    rc = lib.dgxm_attn_fwd_routed(ctypes.byref(d), FAKE, FAKE, FAKE, None, None, None, peers, 9, 0, 8,
                                  0, None, None)
    _status(lib, rc, 1, "out of range")
    rc = lib.dgxm_attn_fwd_routed(ctypes.byref(d), FAKE, FAKE, FAKE, None, None, None, peers, 2, 0, 5,
                                  0, None, None)
    _status(lib, rc, 1, "does not cover")


def _a2a(**kw):
    from dgx_monarch_b200.ulysses import a2a_desc

    args = {"n_tensors": 1, "world": 2, "rank": 0, "batch": 1, "seq_local": 4, "heads": 4, "head_dim": 128,
            "strides": [(4 * 4 * 128, 4 * 128, 128)]}
    args.update(kw)
    import torch

    return a2a_desc(args["n_tensors"], args["world"], args["rank"], args["batch"], args["seq_local"],
                    args["heads"], args["head_dim"], torch.bfloat16, args["strides"], args.get("seg0", 0))


@pytest.mark.parametrize("kw,code,needle", [
    ({"n_tensors": 0}, 1, "1..3 tensors"),
    ({"heads": 3}, 1, "not divisible"),
    ({"head_dim": 4}, 1, "multiple of 16"),
    ({"rank": 2}, 1, "out of range"),
    ({"seq_local": 0}, 0, ""),
])
def test_scatter_argument_checks(lib, kw, code, needle):
    d = _a2a(**kw)
    src = (ctypes.c_void_p * 1)(FAKE)
    dst = (ctypes.c_void_p * 2)(FAKE, FAKE)
    _status(lib, lib.dgxm_ulysses_scatter(ctypes.byref(d), src, dst, None), code, needle)


@pytest.mark.parametrize("seg0,txt_rows,front,needle", [
    (1, 2, 1, "seg0 = 0"),
    (0, -1, 1, "out of range"),
    (0, 2, 2, "out of range"),
])
def test_joint_scatter_argument_checks(lib, seg0, txt_rows, front, needle):
    d = _a2a(seg0=seg0)
    src = (ctypes.c_void_p * 1)(FAKE)
    dst = (ctypes.c_void_p * 2)(FAKE, FAKE)
    txt = (ctypes.c_void_p * 1)(FAKE)
    strides = (ctypes.c_int64 * 3)(2 * 4 * 128, 4 * 128, 128)
    rc = lib.dgxm_ulysses_scatter_joint(ctypes.byref(d), txt_rows, front, txt, strides, src, dst, None)
    _status(lib, rc, 1, needle)


def test_merge_combine_copy_and_comm_checks(lib):
    parts = (ctypes.c_void_p * 2)(FAKE, FAKE)
    lses = (ctypes.c_void_p * 2)(FAKE, FAKE)
    _status(lib, lib.dgxm_lse_merge(1, 8, 2, 64, 2, parts, 3, lses, FAKE, 0, None, None), 2, "head_dim 64")
    _status(lib, lib.dgxm_lse_merge(1, 8, 2, 128, 0, parts, 3, lses, FAKE, 0, None, None), 1, "parts")
    _status(lib, lib.dgxm_lse_merge(1, 0, 2, 128, 2, parts, 3, lses, None, 0, None, None), 0, "")
    _status(lib, lib.dgxm_cfg_combine(FAKE, FAKE, -1, 3, 2.0, FAKE, None), 1, "negative")
    _status(lib, lib.dgxm_cfg_combine(FAKE, FAKE, 64, 2, 2.0, FAKE, None), 2, "dtype 2")
    _status(lib, lib.dgxm_cfg_combine(FAKE, FAKE + 4, 64, 3, 2.0, FAKE, None), 1, "aligned")
    _status(lib, lib.dgxm_cfg_combine(None, None, 0, 3, 2.0, None, None), 0, "")
    _status(lib, lib.dgxm_copy_2d(FAKE, 16, FAKE, 64, 32, 4, None), 1, "pitches")
    _status(lib, lib.dgxm_copy_2d(None, 16, None, 16, 0, 4, None), 0, "")
    handle = ctypes.c_void_p()
    _status(lib, lib.dgxm_comm_create(0, 0, 1024, 1, ctypes.byref(handle)), 1, "out of range")
    _status(lib, lib.dgxm_comm_create(2, 2, 1024, 1, ctypes.byref(handle)), 1, "out of range")
    _status(lib, lib.dgxm_comm_create(0, 2, -1, 1, ctypes.byref(handle)), 1, "negative")
    _status(lib, lib.dgxm_comm_barrier(None, None), 1, "NULL comm")
