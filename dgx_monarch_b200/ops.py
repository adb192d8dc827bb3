"""Torch-facing wrappers over the C ABI: attention forward and the LSE merge.

Tensors stay in the reference's (batch, rows, heads, head_dim) layout
(adapters/cudnn_ring_attention.py:66-89); only pointers, strides and the
current CUDA stream cross into libdgxm_sp.so.  There is no CPU path: a
non-CUDA tensor or a missing library raises.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_FP8 = getattr(torch, "float8_e4m3fn", None)


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    if dtype == torch.float32:
        return _lib.DTYPE_F32
    if _FP8 is not None and dtype == _FP8:
        return _lib.DTYPE_E4M3
    raise TypeError(f"dtype {dtype} is not supported by the B200 attention path")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t.device.type != "cuda":
            raise RuntimeError("the B200 attention path runs on CUDA tensors only "
                               f"(got a tensor on {t.device}); there is no CPU fallback")
        if t.device != dev:
            raise RuntimeError("all tensors of one call must live on the same CUDA device")
    return dev


def attn_desc(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
              lse: torch.Tensor | None, softmax_scale: float | None = None,
              safe_order: bool = False) -> _lib.AttnDesc:
    """The C descriptor of one attention call over (B, L, H, D) tensors."""
    b, lq, h, d = q.shape
    _, lk, hkv, _ = k.shape
    desc = _lib.AttnDesc()
    desc.batch, desc.q_len, desc.kv_len = b, lq, lk
    desc.q_heads, desc.kv_heads, desc.head_dim = h, hkv, d
    desc.in_dtype = _dtype_code(q.dtype)
    desc.out_dtype = _dtype_code(out.dtype)
    desc.q_stride[:] = [q.stride(0), q.stride(1), q.stride(2)]
    desc.k_stride[:] = [k.stride(0), k.stride(1), k.stride(2)]
    desc.v_stride[:] = [v.stride(0), v.stride(1), v.stride(2)]
    desc.o_stride[:] = [out.stride(0), out.stride(1), out.stride(2)]
    if lse is not None:
        desc.lse_stride[:] = [lse.stride(0), lse.stride(1), lse.stride(2)]
    desc.softmax_scale = float(softmax_scale) if softmax_scale else 1.0 / math.sqrt(d)
    desc.flags = _lib.ATTN_SAFE_ORDER if safe_order else 0
    return desc


def attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                  softmax_scale: float | None = None,
                  out_dtype: torch.dtype = torch.bfloat16,
                  q_descale: torch.Tensor | None = None,
                  k_descale: torch.Tensor | None = None,
                  v_descale: torch.Tensor | None = None,
                  out: torch.Tensor | None = None,
                  lse: torch.Tensor | None = None,
                  return_lse: bool = True,
                  safe_order: bool = False) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Non-causal attention over (B, L, H, D) tensors; returns (out, lse).

    ``lse`` is fp32 (B, H, Lq), the natural-log log-sum-exp of the scaled
    logits, as the reference's ring processor contract requires.  bf16 inputs
    run the bf16 tensor-core path; float8_e4m3fn inputs need fp32 descale
    vectors (one per query head for q, one per key/value head for k and v).
    """
    dev = _require_cuda(q, k, v)
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k and v must be 4-D (batch, rows, heads, head_dim)")
    b, lq, h, d = q.shape
    _, lk, hkv, _ = k.shape
    if k.shape != v.shape or k.shape[0] != b or k.shape[3] != d:
        raise ValueError(f"k/v shape {tuple(k.shape)}/{tuple(v.shape)} does not match q {tuple(q.shape)}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("q, k and v must share one dtype")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.stride(3) != 1:
            raise ValueError(f"{name} must have a contiguous head_dim")
    if out is None:
        out = torch.empty((b, lq, h, d), device=dev, dtype=out_dtype)
    if lse is None and return_lse:
        lse = torch.empty((b, h, lq), device=dev, dtype=torch.float32)
    desc = attn_desc(q, k, v, out, lse, softmax_scale, safe_order)
    lib = _lib.load()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.dgxm_attn_fwd(ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                               _ptr(q_descale), _ptr(k_descale), _ptr(v_descale),
                               out.data_ptr(), _ptr(lse), stream)
    _lib.check(rc, "dgxm_attn_fwd")
    return out, lse


def lse_merge(parts_out: list[torch.Tensor], parts_lse: list[torch.Tensor], *,
              out_dtype: torch.dtype = torch.bfloat16,
              out: torch.Tensor | None = None,
              lse_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge per-block (out_i (B,L,H,D), lse_i fp32 (B,H,L)) into the full result."""
    if not parts_out or len(parts_out) != len(parts_lse):
        raise ValueError("lse_merge needs one lse tensor per output part")
    dev = _require_cuda(*parts_out, *parts_lse)
    b, rows, heads, d = parts_out[0].shape
    for o, l in zip(parts_out, parts_lse):
        if o.shape != parts_out[0].shape or o.dtype != parts_out[0].dtype or not o.is_contiguous():
            raise ValueError("merge parts must be contiguous and share shape and dtype")
        if l.shape != (b, heads, rows) or l.dtype != torch.float32 or not l.is_contiguous():
            raise ValueError("merge lse parts must be contiguous fp32 (B, H, L)")
    if out is None:
        out = torch.empty((b, rows, heads, d), device=dev, dtype=out_dtype)
    if lse_out is None:
        lse_out = torch.empty((b, heads, rows), device=dev, dtype=torch.float32)
    n = len(parts_out)
    outs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in parts_out])
    lses = (ctypes.c_void_p * n)(*[t.data_ptr() for t in parts_lse])
    lib = _lib.load()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.dgxm_lse_merge(b, rows, heads, d, n, outs, _dtype_code(parts_out[0].dtype), lses,
                                out.data_ptr(), _dtype_code(out.dtype), lse_out.data_ptr(), stream)
    _lib.check(rc, "dgxm_lse_merge")
    return out, lse_out
