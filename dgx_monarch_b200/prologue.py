"""Torch-facing wrappers: fused Q/K norm + RoPE + Ulysses scatter, RoPE
tables, and per-head e4m3 quantisation."""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import _require_cuda


def rope_table(positions: torch.Tensor, axes_dim: list[int], theta: float = 10000.0) -> torch.Tensor:
    """(rows, 64, 2) fp32 cos/sin table for multi-axis RoPE over head_dim 128.

    positions: (rows, n_axes) coordinates of each local token (e.g. (t, h, w)
    for video, (0, h, w) / (0, 0, 0) for Flux image / text tokens); axis a owns
    axes_dim[a] / 2 consecutive rotation pairs with frequencies
    theta^(-2i / axes_dim[a]).  The angle is computed in float64 and rounded
    once (the standard N-D rotary embedding).
    """
    if sum(axes_dim) != 128:
        raise ValueError(f"axes_dim {axes_dim} must sum to the head dimension 128")
    cols = []
    pos = positions.to(torch.float64)
    for a, dim in enumerate(axes_dim):
        omega = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64, device=pos.device) / dim))
        cols.append(pos[:, a:a + 1] * omega[None, :])
    ang = torch.cat(cols, dim=1)
    return torch.stack((torch.cos(ang), torch.sin(ang)), dim=-1).to(torch.float32).contiguous()


def qkv_prologue_scatter(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, dst_ptrs: list[list[int]],
                         *, world: int, rank: int, norm_mode: int = _lib.NORM_NONE,
                         norm_q_w: torch.Tensor | None = None, norm_k_w: torch.Tensor | None = None,
                         eps: float = 1e-6, rope: torch.Tensor | None = None, seg0: int = 0,
                         stream=None) -> None:
    """Norm + RoPE this rank's (B, Ls, H, 128) q/k rows and scatter q/k/v
    head slices to dst_ptrs[t][r] (rank-major, or joint order with seg0)."""
    _require_cuda(q, k, v, norm_q_w, norm_k_w, rope)
    b, ls, h, d = q.shape
    for t in (q, k, v):
        if t.shape != q.shape or t.dtype != torch.bfloat16 or t.stride(3) != 1:
            raise ValueError("prologue tensors must be bf16 (B, Ls, H, 128) with contiguous head_dim")
    if rope is not None and (rope.dtype != torch.float32 or not rope.is_contiguous()
                             or rope.shape[-2:] != (64, 2) or rope.shape[-3] != ls):
        raise ValueError("rope must be a contiguous fp32 (Ls, 64, 2) or (B, Ls, 64, 2) table")
    desc = _lib.PrologueDesc()
    desc.world, desc.rank, desc.batch, desc.seq_local = world, rank, b, ls
    desc.heads, desc.head_dim, desc.norm_mode, desc.eps = h, d, norm_mode, eps
    for i, t in enumerate((q, k, v)):
        desc.src_stride[i][0], desc.src_stride[i][1], desc.src_stride[i][2] = t.stride(0), t.stride(1), t.stride(2)
    desc.rope_batch_stride = 0 if rope is None or rope.ndim == 3 else rope.stride(0)
    desc.seg0 = seg0
    src = (ctypes.c_void_p * 3)(q.data_ptr(), k.data_ptr(), v.data_ptr())
    dst = (ctypes.c_void_p * (3 * world))(*[p for row in dst_ptrs for p in row])
    stream = stream or torch.cuda.current_stream(q.device)
    ptr = lambda t: None if t is None else t.data_ptr()
    _lib.check(_lib.load().dgxm_qkv_prologue_scatter(ctypes.byref(desc), src, ptr(norm_q_w), ptr(norm_k_w),
                                                     ptr(rope), dst, stream.cuda_stream),
               "dgxm_qkv_prologue_scatter")


def qkv_gemm_prologue_scatter(x: torch.Tensor, w_qkv: torch.Tensor, dst_ptrs: list[list[int]], *,
                              world: int, rank: int, seq_local: int, row0: int = 0, seg0: int = 0,
                              bias: torch.Tensor | None = None, norm_mode: int = _lib.NORM_NONE,
                              norm_q_w: torch.Tensor | None = None, norm_k_w: torch.Tensor | None = None,
                              eps: float = 1e-6, rope: torch.Tensor | None = None, stream=None) -> None:
    """The QKV Linear of one token stream fused with per-head Q/K RMSNorm,
    RoPE and the sequence->head scatter (dgxm_qkv_gemm_prologue_scatter).

    x: (m, k) or (1, m, k) bf16 rows, contiguous features; w_qkv: the Linear
    weight (3 * heads * 128, k); dst_ptrs[t][r]: rank r's (world * seq_local,
    heads / world, 128) receive tensor t; rope: (seq_local, 64, 2) fp32."""
    _require_cuda(x, w_qkv, bias, norm_q_w, norm_k_w, rope)
    x2 = x.reshape(-1, x.shape[-1]) if x.ndim == 3 else x
    if x.ndim == 3 and x.shape[0] != 1:
        raise ValueError("the fused QKV kernel takes one batch item per call")
    m, k = x2.shape
    n = w_qkv.shape[0]
    if x2.dtype != torch.bfloat16 or w_qkv.dtype != torch.bfloat16 or x2.stride(1) != 1 or not w_qkv.is_contiguous():
        raise ValueError("x and w_qkv must be bf16 with contiguous features")
    if w_qkv.shape[1] != k or n % 384:
        raise ValueError(f"w_qkv {tuple(w_qkv.shape)} is not a (3 * heads * 128, {k}) Linear weight")
    if rope is not None and (rope.dtype != torch.float32 or not rope.is_contiguous()
                             or tuple(rope.shape) != (seq_local, 64, 2)):
        raise ValueError("rope must be a contiguous fp32 (seq_local, 64, 2) table")
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != n or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous bf16 vector of the Linear's outputs")
    desc = _lib.QkvGemmDesc()
    desc.world, desc.rank, desc.m, desc.k = world, rank, m, k
    desc.heads, desc.seq_local, desc.row0, desc.seg0 = n // 384, seq_local, row0, seg0
    desc.norm_mode, desc.eps, desc.x_row_stride = norm_mode, eps, x2.stride(0)
    dst = (ctypes.c_void_p * (3 * world))(*[p for row in dst_ptrs for p in row])
    stream = stream or torch.cuda.current_stream(x.device)
    ptr = lambda t: None if t is None else t.data_ptr()
    _lib.check(_lib.load().dgxm_qkv_gemm_prologue_scatter(
        ctypes.byref(desc), x2.data_ptr(), w_qkv.data_ptr(), ptr(bias), ptr(norm_q_w), ptr(norm_k_w),
        ptr(rope), dst, stream.cuda_stream), "dgxm_qkv_gemm_prologue_scatter")


def qkv_gemm_prologue_scatter_streams(streams: list[dict], dst_ptrs: list[list[int]], *, world: int,
                                      rank: int, seq_local: int, seg0: int = 0,
                                      norm_mode: int = _lib.NORM_NONE, eps: float = 1e-6,
                                      rope: torch.Tensor | None = None, stream=None) -> None:
    """qkv_gemm_prologue_scatter for one or two token streams in one launch
    (dgxm_qkv_gemm_prologue_scatter_streams): a joint block's text and image
    projections share one grid of pair tiles.  Each stream is a dict with
    x, w_qkv, row0 and optionally bias, norm_q_w and norm_k_w, as the
    single-stream call takes them; every head row comes out as that call
    writes it."""
    if not 1 <= len(streams) <= 2:
        raise ValueError(f"{len(streams)} streams (1 or 2)")
    if rope is not None and (rope.dtype != torch.float32 or not rope.is_contiguous()
                             or tuple(rope.shape) != (seq_local, 64, 2)):
        raise ValueError("rope must be a contiguous fp32 (seq_local, 64, 2) table")
    arr = (_lib.QkvStream * len(streams))()
    ptr = lambda t: None if t is None else t.data_ptr()
    k = n = None
    keep = []  # the 2-D views passed by pointer stay alive until the launch
    for i, st in enumerate(streams):
        x, w_qkv = st["x"], st["w_qkv"]
        bias, nq, nk = st.get("bias"), st.get("norm_q_w"), st.get("norm_k_w")
        _require_cuda(x, w_qkv, bias, nq, nk, rope)
        x2 = x.reshape(-1, x.shape[-1]) if x.ndim == 3 else x
        if x.ndim == 3 and x.shape[0] != 1:
            raise ValueError("the fused QKV kernel takes one batch item per stream")
        if x2.dtype != torch.bfloat16 or w_qkv.dtype != torch.bfloat16 or x2.stride(1) != 1 \
                or not w_qkv.is_contiguous():
            raise ValueError("x and w_qkv must be bf16 with contiguous features")
        if k is None:
            k, n = x2.shape[1], w_qkv.shape[0]
        if x2.shape[1] != k or tuple(w_qkv.shape) != (n, k) or n % 384:
            raise ValueError("the streams' inputs and Linear weights must share (3 * heads * 128, k)")
        if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != n or not bias.is_contiguous()):
            raise ValueError("bias must be a contiguous bf16 vector of the Linear's outputs")
        keep.append(x2)
        arr[i].x, arr[i].w_qkv, arr[i].bias = x2.data_ptr(), w_qkv.data_ptr(), ptr(bias)
        arr[i].norm_q_w, arr[i].norm_k_w = ptr(nq), ptr(nk)
        arr[i].x_row_stride, arr[i].m, arr[i].row0 = x2.stride(0), x2.shape[0], int(st.get("row0", 0))
    desc = _lib.QkvGemmDesc()
    desc.world, desc.rank, desc.k = world, rank, k
    desc.heads, desc.seq_local, desc.seg0 = n // 384, seq_local, seg0
    desc.norm_mode, desc.eps = norm_mode, eps
    dst = (ctypes.c_void_p * (3 * world))(*[p for row in dst_ptrs for p in row])
    stream = stream or torch.cuda.current_stream(streams[0]["x"].device)
    _lib.check(_lib.load().dgxm_qkv_gemm_prologue_scatter_streams(
        ctypes.byref(desc), len(streams), arr, ptr(rope), dst, stream.cuda_stream),
        "dgxm_qkv_gemm_prologue_scatter_streams")


def quantize_e4m3_per_head(x: torch.Tensor, out: torch.Tensor | None = None,
                           descale: torch.Tensor | None = None, stream=None,
                           keep: torch.Tensor | None = None):
    """(e4m3 values, fp32 per-head descale = absmax / 448) of a bf16 (B, L, H, 128) tensor.

    keep: optional row keep bits (ops.keep_bits: int32 words, (W,) for every
    batch row or (B, W)); a cleared row does not count toward the absmax, so
    the scale is the one the real rows alone give."""
    _require_cuda(x, out, descale, keep)
    b, l, h, d = x.shape
    if x.dtype != torch.bfloat16 or x.stride(3) != 1:
        raise ValueError("quantisation input must be bf16 with contiguous head_dim")
    if out is None:
        out = torch.empty(b, l, h, d, device=x.device, dtype=torch.float8_e4m3fn)
    elif tuple(out.shape) != (b, l, h, d) or out.dtype != torch.float8_e4m3fn or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous float8_e4m3fn tensor of shape {(b, l, h, d)}")
    if descale is None:
        descale = torch.empty(h, device=x.device, dtype=torch.float32)
    elif descale.numel() != h or descale.dtype != torch.float32 or not descale.is_contiguous():
        raise ValueError(f"descale must be a contiguous fp32 vector of {h} heads")
    stride = (ctypes.c_int64 * 3)(x.stride(0), x.stride(1), x.stride(2))
    stream = stream or torch.cuda.current_stream(x.device)
    if keep is None:
        _lib.check(_lib.load().dgxm_quantize_e4m3_per_head(b, l, h, d, x.data_ptr(), stride,
                                                           out.data_ptr(), descale.data_ptr(),
                                                           stream.cuda_stream),
                   "dgxm_quantize_e4m3_per_head")
        return out, descale
    words = (l + 31) // 32
    if (keep.dtype != torch.int32 or keep.stride(-1) != 1 or keep.shape[-1] != words
            or keep.ndim not in (1, 2) or (keep.ndim == 2 and keep.shape[0] != b)):
        raise ValueError(f"keep must be int32 keep bits of shape ({words},) or ({b}, {words})")
    _lib.check(_lib.load().dgxm_quantize_e4m3_per_head_masked(
        b, l, h, d, x.data_ptr(), stride, keep.data_ptr(), keep.stride(0) if keep.ndim == 2 else 0,
        out.data_ptr(), descale.data_ptr(), stream.cuda_stream), "dgxm_quantize_e4m3_per_head_masked")
    return out, descale


def quantize_e4m3_per_head_many(items, stream=None):
    """Quantise up to three bf16 (B, L, H, 128) tensors in the same launches
    (dgxm_quantize_e4m3_per_head_batch): items are (x, out, descale, keep)
    tuples as quantize_e4m3_per_head takes them (out, descale and keep may be
    None).  Returns [(e4m3 values, fp32 descale)] in item order."""
    items = list(items)
    if not 1 <= len(items) <= 3:
        raise ValueError("quantisation batches take 1 to 3 tensors")
    arr = (_lib.QuantItem * len(items))()
    results = []
    dev = None
    for slot, (x, out, descale, keep) in zip(arr, items):
        d = _require_cuda(x, out, descale, keep)
        if dev is not None and d != dev:
            raise RuntimeError("every tensor of one quantisation batch must live on one device")
        dev = d
        b, l, h, hd = x.shape
        if x.dtype != torch.bfloat16 or x.stride(3) != 1:
            raise ValueError("quantisation input must be bf16 with contiguous head_dim")
        if out is None:
            out = torch.empty(b, l, h, hd, device=x.device, dtype=torch.float8_e4m3fn)
        elif tuple(out.shape) != (b, l, h, hd) or out.dtype != torch.float8_e4m3fn or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous float8_e4m3fn tensor of shape {(b, l, h, hd)}")
        if descale is None:
            descale = torch.empty(h, device=x.device, dtype=torch.float32)
        elif descale.numel() != h or descale.dtype != torch.float32 or not descale.is_contiguous():
            raise ValueError(f"descale must be a contiguous fp32 vector of {h} heads")
        words = (l + 31) // 32
        if keep is not None and (keep.dtype != torch.int32 or keep.stride(-1) != 1 or keep.shape[-1] != words
                                 or keep.ndim not in (1, 2) or (keep.ndim == 2 and keep.shape[0] != b)):
            raise ValueError(f"keep must be int32 keep bits of shape ({words},) or ({b}, {words})")
        slot.batch, slot.rows, slot.heads, slot.head_dim = b, l, h, hd
        slot.x = x.data_ptr()
        slot.stride[:] = [x.stride(0), x.stride(1), x.stride(2)]
        slot.keep = None if keep is None else keep.data_ptr()
        slot.keep_batch_stride = keep.stride(0) if keep is not None and keep.ndim == 2 else 0
        slot.out = out.data_ptr()
        slot.descale = descale.data_ptr()
        results.append((out, descale))
    stream = stream or torch.cuda.current_stream(dev)
    _lib.check(_lib.load().dgxm_quantize_e4m3_per_head_batch(len(items), arr, stream.cuda_stream),
               "dgxm_quantize_e4m3_per_head_batch")
    return results
