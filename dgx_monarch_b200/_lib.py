"""ctypes binding of libdgxm_sp.so (the C ABI declared in include/dgxm_sp.h).

This is the binding a maintainer of the reference would add: plain pointers,
sizes and a stream handle, int status codes turned into Python exceptions.
The library must be built (``python -m dgx_monarch_b200._build``); there is
no fallback when it is missing.
"""
from __future__ import annotations

import ctypes
import threading

from ._build import LIB_PATH

DGXM_OK = 0
DGXM_ERR_INVALID = 1
DGXM_ERR_UNSUPPORTED = 2
DGXM_ERR_CUDA = 3
DGXM_ERR_TIMEOUT = 4
DGXM_ERR_STATE = 5

DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_E4M3 = 2
DTYPE_F32 = 3

ATTN_SAFE_ORDER = 1
ATTN_ONE_CTA = 2  # DGXM_ATTN_ONE_CTA
ATTN_P_CHUNKS_SHIFT = 4  # DGXM_ATTN_P_CHUNKS(n) = n << 4


class DgxmError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, func: str, message: str) -> None:
        super().__init__(f"{func} failed with status {code}: {message}")
        self.code = code
        self.func = func


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("q_len", ctypes.c_int32),
        ("kv_len", ctypes.c_int32),
        ("q_heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("in_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("q_stride", ctypes.c_int64 * 3),
        ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3),
        ("o_stride", ctypes.c_int64 * 3),
        ("lse_stride", ctypes.c_int64 * 3),
        ("softmax_scale", ctypes.c_float),
        ("flags", ctypes.c_int32),
    ]


MAX_WORLD = 8
IPC_HANDLE_BYTES = 64


class A2ADesc(ctypes.Structure):
    _fields_ = [
        ("n_tensors", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("seq_local", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("src_stride", (ctypes.c_int64 * 3) * 3),
        ("seg0", ctypes.c_int32),
    ]


MAX_BIAS_GROUPS = 8


class AttnExtras(ctypes.Structure):
    _fields_ = [
        ("key_keep", ctypes.c_void_p),
        ("key_keep_batch_stride", ctypes.c_int64),
        ("query_keep", ctypes.c_void_p),
        ("query_keep_batch_stride", ctypes.c_int64),
        ("n_bias_groups", ctypes.c_int32),
        ("bias_row_begin", ctypes.c_int32 * MAX_BIAS_GROUPS),
        ("bias_row_end", ctypes.c_int32 * MAX_BIAS_GROUPS),
        ("bias", ctypes.c_void_p * MAX_BIAS_GROUPS),
        ("bias_stride", (ctypes.c_int64 * 3) * MAX_BIAS_GROUPS),
        ("bias_keys", ctypes.c_int32 * MAX_BIAS_GROUPS),
    ]


class AttnRoute(ctypes.Structure):
    _fields_ = [
        ("o_peers", ctypes.c_void_p * 8),
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("seq_local", ctypes.c_int32),
        ("seg0", ctypes.c_int32),
        ("txt_rows", ctypes.c_int32),
        ("txt_front", ctypes.c_int32),
        ("txt_peers", ctypes.c_void_p * 8),
    ]


class SeqGatherDesc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("seq_local", ctypes.c_int32),
        ("orig_len", ctypes.c_int32),
        ("row_bytes", ctypes.c_int32),
        ("src_batch_stride", ctypes.c_int64),
        ("src_row_stride", ctypes.c_int64),
    ]


class QkvGemmDesc(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("m", ctypes.c_int32),
        ("k", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("seq_local", ctypes.c_int32),
        ("row0", ctypes.c_int32),
        ("seg0", ctypes.c_int32),
        ("norm_mode", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("x_row_stride", ctypes.c_int64),
    ]


class QkvStream(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p),
        ("w_qkv", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("norm_q_w", ctypes.c_void_p),
        ("norm_k_w", ctypes.c_void_p),
        ("x_row_stride", ctypes.c_int64),
        ("m", ctypes.c_int32),
        ("row0", ctypes.c_int32),
    ]


NORM_NONE, NORM_HIDDEN, NORM_HEAD = 0, 1, 2


class QuantItem(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("rows", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("stride", ctypes.c_int64 * 3),
        ("keep", ctypes.c_void_p),
        ("keep_batch_stride", ctypes.c_int64),
        ("out", ctypes.c_void_p),
        ("descale", ctypes.c_void_p),
    ]


class PrologueDesc(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("seq_local", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("norm_mode", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("src_stride", (ctypes.c_int64 * 3) * 3),
        ("rope_batch_stride", ctypes.c_int64),
        ("seg0", ctypes.c_int32),
    ]


# Every symbol include/dgxm_sp.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "dgxm_abi_version": (ctypes.c_int, []),
    "dgxm_last_error_message": (ctypes.c_char_p, []),
    "dgxm_device_error": (ctypes.c_int, [ctypes.c_int]),
    "dgxm_attn_fwd": (ctypes.c_int, [ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "dgxm_lse_merge": (ctypes.c_int, [_I32, _I32, _I32, _I32, _I32, ctypes.POINTER(_P), _I32,
                                      ctypes.POINTER(_P), _P, _I32, _P, _P]),
    "dgxm_comm_create": (ctypes.c_int, [_I32, _I32, ctypes.c_int64, ctypes.c_uint64,
                                        ctypes.POINTER(_P)]),
    "dgxm_comm_export": (ctypes.c_int, [_P, _P]),
    "dgxm_comm_import": (ctypes.c_int, [_P, _P]),
    "dgxm_comm_window": (ctypes.c_int, [_P, _I32, ctypes.POINTER(_P)]),
    "dgxm_comm_bytes": (ctypes.c_int64, [_P]),
    "dgxm_comm_generation": (ctypes.c_uint64, [_P]),
    "dgxm_comm_barrier": (ctypes.c_int, [_P, _P]),
    "dgxm_comm_set_timeout": (ctypes.c_int, [_P, _I32]),
    "dgxm_comm_allgather": (ctypes.c_int, [_P, _P, ctypes.c_int64, ctypes.c_int64, _P]),
    "dgxm_comm_destroy": (ctypes.c_int, [_P]),
    "dgxm_ulysses_scatter": (ctypes.c_int, [ctypes.POINTER(A2ADesc), ctypes.POINTER(_P),
                                            ctypes.POINTER(_P), _P]),
    "dgxm_ulysses_scatter_joint": (ctypes.c_int, [ctypes.POINTER(A2ADesc), ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_int64),
                                                  ctypes.POINTER(_P), ctypes.POINTER(_P), _P]),
    "dgxm_ulysses_gather": (ctypes.c_int, [ctypes.POINTER(A2ADesc), _P, ctypes.POINTER(_P), _P]),
    "dgxm_attn_fwd_ext": (ctypes.c_int, [ctypes.POINTER(AttnDesc), ctypes.POINTER(AttnExtras),
                                         ctypes.POINTER(AttnRoute), _P, _P, _P, _P, _P, _P, _P, _P,
                                         _P]),
    "dgxm_attn_fwd_routed": (ctypes.c_int, [ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P, _P,
                                            ctypes.POINTER(_P), _I32, _I32, _I32, _I32, _P, _P]),
    "dgxm_qkv_prologue_scatter": (ctypes.c_int, [ctypes.POINTER(PrologueDesc), ctypes.POINTER(_P),
                                                 _P, _P, _P, ctypes.POINTER(_P), _P]),
    "dgxm_quantize_e4m3_per_head": (ctypes.c_int, [_I32, _I32, _I32, _I32, _P,
                                                   ctypes.POINTER(ctypes.c_int64), _P, _P, _P]),
    "dgxm_quantize_e4m3_per_head_batch": (ctypes.c_int, [_I32, ctypes.POINTER(QuantItem), _P]),
    "dgxm_quantize_e4m3_per_head_masked": (ctypes.c_int, [_I32, _I32, _I32, _I32, _P,
                                                          ctypes.POINTER(ctypes.c_int64), _P,
                                                          ctypes.c_int64, _P, _P, _P]),
    "dgxm_ring_window_bytes": (ctypes.c_int64, [ctypes.POINTER(AttnDesc)]),
    "dgxm_ring_workspace_bytes": (ctypes.c_int64, [ctypes.POINTER(AttnDesc), _I32]),
    "dgxm_ring_attn_fwd": (ctypes.c_int, [_P, ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P, _P,
                                          ctypes.c_int64, _P]),
    "dgxm_ring_attn_fwd_fp8": (ctypes.c_int, [_P, ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P, _P, _P,
                                              _P, _P, ctypes.c_int64, _P]),
    "dgxm_ring_noalloc_max_bytes": (ctypes.c_int64, []),
    "dgxm_ring_attn_fwd_noalloc": (ctypes.c_int, [_P, ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P,
                                                  _P]),
    "dgxm_full_context_window_bytes": (ctypes.c_int64, [ctypes.POINTER(AttnDesc), _I32]),
    "dgxm_qkv_gemm_prologue_scatter": (ctypes.c_int, [ctypes.POINTER(QkvGemmDesc), _P, _P, _P, _P, _P, _P,
                                                      _P, _P]),
    "dgxm_qkv_gemm_prologue_scatter_streams": (ctypes.c_int, [ctypes.POINTER(QkvGemmDesc), _I32,
                                                              ctypes.POINTER(QkvStream), _P, _P, _P]),
    "dgxm_copy_2d": (ctypes.c_int, [_P, ctypes.c_int64, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _P]),
    "dgxm_cfg_combine": (ctypes.c_int, [_P, _P, ctypes.c_int64, _I32, ctypes.c_double, _P, _P]),
    "dgxm_seq_allgather": (ctypes.c_int, [_P, ctypes.POINTER(SeqGatherDesc), _P, ctypes.c_int64, _P]),
    "dgxm_seq_gather_store": (ctypes.c_int, [ctypes.POINTER(SeqGatherDesc), _I32, _I32, _P,
                                             ctypes.POINTER(_P), _P]),
    "dgxm_kv_gather_store": (ctypes.c_int, [ctypes.POINTER(AttnDesc), _I32, _I32, _P, _P,
                                            ctypes.POINTER(_P), ctypes.POINTER(_P), _P]),
    "dgxm_shared_amax_scale": (ctypes.c_int, [_P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              _I32, ctypes.c_float, _P, _P, _P]),
    "dgxm_full_context_attn_fwd": (ctypes.c_int, [_P, ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P,
                                                  _P]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load(path=None) -> ctypes.CDLL:
    """Load the library once and attach the declared signatures."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = str(path or LIB_PATH)
        try:
            lib = ctypes.CDLL(target)
        except OSError as exc:
            raise RuntimeError(
                f"libdgxm_sp.so could not be loaded from {target}: {exc}. Build it with "
                "`python -m dgx_monarch_b200._build` (nvcc, sm_100a); the attention path has "
                "no CPU fallback.") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if path is None:
            _lib = lib
        return lib


def check(code: int, func: str) -> None:
    if code != DGXM_OK:
        msg = load().dgxm_last_error_message()
        raise DgxmError(code, func, msg.decode(errors="replace") if msg else "")


# Bits of the device error word (csrc/common.h).
ERR_PRODUCER_TIMEOUT, ERR_MMA_TIMEOUT, ERR_SOFTMAX_TIMEOUT, ERR_EPILOGUE_TIMEOUT, ERR_PEER_TIMEOUT = 1, 2, 4, 8, 16


def device_error(clear: bool = True) -> int:
    """The device error word (bounded waits that expired); 0 when clean."""
    value = load().dgxm_device_error(1 if clear else 0)
    if value < 0:
        check(-value, "dgxm_device_error")
    return value
