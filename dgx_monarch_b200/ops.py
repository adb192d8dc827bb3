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
    if dtype == torch.float16:
        return _lib.DTYPE_F16
    if dtype == torch.float32:
        return _lib.DTYPE_F32
    if _FP8 is not None and dtype == _FP8:
        return _lib.DTYPE_E4M3
    raise TypeError(f"dtype {dtype} is not supported by the B200 attention path")


def out16_dtype(in_dtype: torch.dtype) -> torch.dtype:
    """The 16-bit output format of an attention over `in_dtype` inputs: fp16
    for fp16, bf16 for bf16 and e4m3."""
    return torch.float16 if in_dtype == torch.float16 else torch.bfloat16


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device | None:
    """All given tensors (None skipped) are CUDA tensors on one device, which
    is returned (None when no tensor is given): no host pointer, nor another
    GPU's, ever reaches a kernel."""
    given = [t for t in tensors if t is not None]
    if not given:
        return None
    dev = given[0].device
    for t in given:
        if t.device.type != "cuda":
            raise RuntimeError("the B200 attention path runs on CUDA tensors only "
                               f"(got a tensor on {t.device}); there is no CPU fallback")
        if t.device != dev:
            raise RuntimeError("all tensors of one call must live on the same CUDA device")
    return dev


def _require_on(device: torch.device, *tensors: torch.Tensor | None) -> None:
    """Like _require_cuda, and the device is the one the operation was built for."""
    dev = _require_cuda(*tensors)
    if dev is None:
        return
    device = torch.device(device)
    want = device.index if device.index is not None else torch.cuda.current_device()
    if dev.index != want:
        raise RuntimeError(f"a tensor on {dev} was passed to an operation set up on cuda:{want}")


def kernel_head_dim(head_dim: int, *, fp8: bool = False, ring: bool = False) -> int:
    """The head dimension a caller's head_dim runs at: 64 for head
    dimensions up to 64 on 16-bit inputs (a native kernel), else 128.  A
    smaller head_dim is zero-padded up to it, which is exact.  The e4m3
    kernel and the ring's merge run 128 only."""
    return 64 if head_dim <= 64 and not fp8 and not ring else 128


def check_attn_buffers(q: torch.Tensor, k: torch.Tensor, *, out: torch.Tensor | None = None,
                       lse: torch.Tensor | None = None, q_descale: torch.Tensor | None = None,
                       k_descale: torch.Tensor | None = None,
                       v_descale: torch.Tensor | None = None) -> None:
    """Caller-given buffers of one attention call cover what the kernel touches:
    out (B, Lq, H, D) with a contiguous head_dim, lse fp32 (B, H, Lq), one fp32
    descale per query head (q) or key/value head (k, v), all on q's device."""
    b, lq, h, d = q.shape
    hkv = k.shape[2]
    _require_on(q.device, out, lse, q_descale, k_descale, v_descale)
    if out is not None and (tuple(out.shape) != (b, lq, h, d) or out.stride(3) != 1):
        raise ValueError(f"out {tuple(out.shape)} is not a {(b, lq, h, d)} tensor with contiguous head_dim")
    if lse is not None and (tuple(lse.shape) != (b, h, lq) or lse.dtype != torch.float32):
        raise ValueError(f"lse {tuple(lse.shape)} {lse.dtype} is not an fp32 {(b, h, lq)} tensor")
    for name, scale, n in (("q_descale", q_descale, h), ("k_descale", k_descale, hkv),
                           ("v_descale", v_descale, hkv)):
        if scale is not None and (scale.dtype != torch.float32 or scale.numel() != n
                                  or not scale.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous fp32 vector of {n} heads")


_P_CHUNKS = 0  # 0: the library's default release of P per 128-key block


def set_p_chunks(chunks: int) -> None:
    """Release each block's probabilities to the tensor core in `chunks` parts
    in every attention call this process makes from now on
    (DGXM_ATTN_P_CHUNKS): 1 is the single release, kept as a cross-check; 0,
    2 and 4 select the library default (4 chunks; 2 for e4m3 inputs)."""
    global _P_CHUNKS
    if chunks not in (0, 1, 2, 4):
        raise ValueError(f"P is released in 1, 2 or 4 chunks, not {chunks}")
    _P_CHUNKS = chunks


_CTA_PAIR = True  # 16-bit head-dim-128 attention on CTA pairs (False: DGXM_ATTN_ONE_CTA)


def set_cta_pair(on: bool) -> None:
    """Run the 16-bit, head-dim-128 attention calls this process makes from
    now on as CTA pairs (the library default: clusters of two CTAs on one
    TPC, each loading half of every K/V block, one thread issuing the M256
    tensor-core products of both) or, with False, on single CTAs
    (DGXM_ATTN_ONE_CTA, kept as a cross-check).  e4m3, head dim 64 and the
    single P release always run on single CTAs."""
    global _CTA_PAIR
    _CTA_PAIR = bool(on)


def attn_flags(safe_order: bool = False) -> int:
    """The descriptor flags of one attention call."""
    return ((_lib.ATTN_SAFE_ORDER if safe_order else 0) | (_P_CHUNKS << _lib.ATTN_P_CHUNKS_SHIFT)
            | (0 if _CTA_PAIR else _lib.ATTN_ONE_CTA))


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
    desc.flags = attn_flags(safe_order)
    return desc


def attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                  softmax_scale: float | None = None,
                  out_dtype: torch.dtype | None = None,
                  q_descale: torch.Tensor | None = None,
                  k_descale: torch.Tensor | None = None,
                  v_descale: torch.Tensor | None = None,
                  out: torch.Tensor | None = None,
                  lse: torch.Tensor | None = None,
                  return_lse: bool = True,
                  safe_order: bool = False) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Non-causal attention over (B, L, H, D) tensors; returns (out, lse).

    ``lse`` is fp32 (B, H, Lq), the natural-log log-sum-exp of the scaled
    logits, as the reference's ring processor contract requires.  bf16 and
    fp16 inputs run the 16-bit tensor-core path in their own format (P too);
    float8_e4m3fn inputs need fp32 descale vectors (one per query head for q,
    one per key/value head for k and v).  out_dtype None is the inputs' 16-bit
    format (bf16 for e4m3); fp32 is the other choice.
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
    check_attn_buffers(q, k, out=out, lse=lse, q_descale=q_descale, k_descale=k_descale, v_descale=v_descale)
    if out is None:
        out = torch.empty((b, lq, h, d), device=dev, dtype=out_dtype or out16_dtype(q.dtype))
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


_KEEP_BITS: dict = {}


def keep_bits(rows: int, drop_rows, device: torch.device) -> torch.Tensor | None:
    """Packed keep bits (int32 words, bit i of word i//32) of `rows` rows with
    `drop_rows` cleared; None when nothing drops.  Cached per layout, like the
    reference's keep index (adapters/usp_pad_exclusion.py:93-126), and range
    checked before any device work."""
    if not drop_rows:
        return None
    key = (rows, tuple(sorted(set(drop_rows))), str(device))
    found = _KEEP_BITS.get(key)
    if found is not None:
        return found
    drop = key[1]
    if drop[-1] >= rows or drop[0] < 0:
        raise ValueError(f"a pad row at index {drop[-1]} was handed to an attention whose axis "
                         f"carries {rows} rows")
    words = (rows + 31) // 32
    bits = [0xFFFFFFFF] * words
    if rows % 32:
        bits[-1] = (1 << (rows % 32)) - 1
    for r in drop:
        bits[r // 32] &= ~(1 << (r % 32)) & 0xFFFFFFFF
    t = torch.tensor([b - (1 << 32) if b >= (1 << 31) else b for b in bits], dtype=torch.int32,
                     device=device)
    if len(_KEEP_BITS) > 64:
        _KEEP_BITS.clear()
    _KEEP_BITS[key] = t
    return t


def attention_fwd_ext(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                      key_keep: torch.Tensor | None = None,
                      query_keep: torch.Tensor | None = None,
                      bias_groups=None,
                      route: dict | None = None,
                      out: torch.Tensor | None = None,
                      out_strides=None,
                      lse: torch.Tensor | None = None,
                      softmax_scale: float | None = None,
                      q_descale=None, k_descale=None, v_descale=None):
    """Attention with keep masks, query-group biases and/or output routing.

    bias_groups: [(row_begin, row_end, bias fp32 (B|1, H|1, Q|1, K') or None)],
    Q the group's row count;
    route: {"o_peers": [ptr...], "world", "rank", "seq_local", "seg0"} with
    out_strides describing the peers' (B, Ls, H_total, D) tensors; optional
    "txt_rows", "txt_front", "txt_peers" route replicated text rows to every
    rank's (B, T, H_total, D) text output (dgxm_attn_route).
    """
    dev = _require_cuda(q, k, v)
    b, lq, h, d = q.shape
    check_attn_buffers(q, k, out=out if route is None else None, lse=lse, q_descale=q_descale,
                       k_descale=k_descale, v_descale=v_descale)
    _require_on(dev, key_keep, query_keep, *[g[2] for g in (bias_groups or [])])
    keep = []
    if out is None and route is None:
        out = torch.empty((b, lq, h, d), device=dev, dtype=out16_dtype(q.dtype))
    probe_out = out if out is not None else torch.empty((1, 1, 1, d), device="meta",
                                                        dtype=out16_dtype(q.dtype))
    desc = attn_desc(q, k, v, probe_out, lse, softmax_scale)
    if out_strides is not None:
        desc.o_stride[:] = list(out_strides)
    ex = _lib.AttnExtras()
    if key_keep is not None:
        ex.key_keep = key_keep.data_ptr()
        ex.key_keep_batch_stride = key_keep.stride(0) if key_keep.ndim == 2 else 0
    if query_keep is not None:
        ex.query_keep = query_keep.data_ptr()
        ex.query_keep_batch_stride = query_keep.stride(0) if query_keep.ndim == 2 else 0
    groups = [g for g in (bias_groups or []) if g[2] is not None]
    if len(groups) > _lib.MAX_BIAS_GROUPS:
        raise ValueError(f"at most {_lib.MAX_BIAS_GROUPS} biased query groups")
    ex.n_bias_groups = len(groups)
    for i, (start, end, bias) in enumerate(groups):
        if bias.dtype != torch.float32 or bias.ndim != 4 or bias.stride(3) != 1:
            raise ValueError("a group bias must be fp32 (B|1, H|1, Q|1, K) with contiguous keys")
        if bias.shape[2] not in (1, end - start):
            raise ValueError(f"a group bias of {bias.shape[2]} query rows over a group of "
                             f"{end - start}")
        keep.append(bias)
        ex.bias_row_begin[i], ex.bias_row_end[i] = int(start), int(end)
        ex.bias[i] = bias.data_ptr()
        ex.bias_stride[i][0] = 0 if bias.shape[0] == 1 else bias.stride(0)
        ex.bias_stride[i][1] = 0 if bias.shape[1] == 1 else bias.stride(1)
        ex.bias_stride[i][2] = 0 if bias.shape[2] == 1 else bias.stride(2)
        ex.bias_keys[i] = bias.shape[3]
    rt = None
    if route is not None:
        rt = _lib.AttnRoute()
        for i, ptr in enumerate(route["o_peers"]):
            rt.o_peers[i] = ptr
        rt.world, rt.rank = route["world"], route["rank"]
        rt.seq_local, rt.seg0 = route["seq_local"], route.get("seg0", 0)
        rt.txt_rows, rt.txt_front = route.get("txt_rows", 0), int(route.get("txt_front", 1))
        for i, ptr in enumerate(route.get("txt_peers", ())):
            rt.txt_peers[i] = ptr
    lib = _lib.load()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.dgxm_attn_fwd_ext(ctypes.byref(desc), ctypes.byref(ex),
                                   ctypes.byref(rt) if rt is not None else None,
                                   q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(q_descale),
                                   _ptr(k_descale), _ptr(v_descale),
                                   out.data_ptr() if out is not None else None, _ptr(lse), stream)
    _lib.check(rc, "dgxm_attn_fwd_ext")
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
    _require_on(dev, out, lse_out)
    if out is None:
        out = torch.empty((b, rows, heads, d), device=dev, dtype=out_dtype)
    elif tuple(out.shape) != (b, rows, heads, d) or not out.is_contiguous():
        raise ValueError(f"merge output {tuple(out.shape)} is not a contiguous {(b, rows, heads, d)} tensor")
    if lse_out is None:
        lse_out = torch.empty((b, heads, rows), device=dev, dtype=torch.float32)
    elif tuple(lse_out.shape) != (b, heads, rows) or lse_out.dtype != torch.float32 or not lse_out.is_contiguous():
        raise ValueError(f"merge lse output must be a contiguous fp32 {(b, heads, rows)} tensor")
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


def copy_2d(dst: int, dpitch: int, src: int, spitch: int, width: int, height: int, stream) -> None:
    """One strided copy-engine transfer (dgxm_copy_2d): height rows of width bytes."""
    _lib.check(_lib.load().dgxm_copy_2d(dst, dpitch, src, spitch, width, height, stream.cuda_stream),
               "dgxm_copy_2d")


class HostStreamedAttention:
    """Attention whose inputs and output live in pinned host memory, streamed
    through the device one head group at a time.

    Heads are independent, so the host->device copy of group g + 1 and the
    device->host copy of group g - 1 (copy engines, one stream each way) run
    while the tensor cores attend group g.  Each group's slice of a
    (B, L, H, D) tensor is one strided copy per tensor.  The result is the
    same bits as one attention_fwd call over the whole tensors.
    """

    def __init__(self, batch: int, q_len: int, kv_len: int, heads: int, kv_heads: int | None = None,
                 head_dim: int = 128, *, device: torch.device, groups: int = 8) -> None:
        kv_heads = heads if kv_heads is None else kv_heads
        if heads % groups or kv_heads % groups:
            raise ValueError(f"{groups} head groups do not split {heads} query / {kv_heads} key-value heads")
        self.shape = (batch, q_len, kv_len, heads, kv_heads, head_dim)
        self.groups, self.device = groups, device
        dt = torch.bfloat16
        self.q = torch.empty(batch, q_len, heads, head_dim, device=device, dtype=dt)
        self.k = torch.empty(batch, kv_len, kv_heads, head_dim, device=device, dtype=dt)
        self.v = torch.empty(batch, kv_len, kv_heads, head_dim, device=device, dtype=dt)
        self.out = torch.empty(batch, q_len, heads, head_dim, device=device, dtype=dt)
        self.copy_in = torch.cuda.Stream(device)
        self.copy_out = torch.cuda.Stream(device)
        self.launches_per_call = groups

    def _slice(self, dst: torch.Tensor, src: torch.Tensor, g: int, stream) -> None:
        """Head group g of a (B, L, H, D) tensor: B * L rows of (H / groups) heads."""
        b, l, h, d = src.shape
        hg = h // self.groups
        elt = src.element_size()
        off = g * hg * d * elt
        copy_2d(dst.data_ptr() + off, h * d * elt, src.data_ptr() + off, h * d * elt, hg * d * elt, b * l, stream)

    def __call__(self, q_host: torch.Tensor, k_host: torch.Tensor, v_host: torch.Tensor,
                 out_host: torch.Tensor) -> torch.Tensor:
        b, lq, lk, h, hkv, d = self.shape
        for t, want in ((q_host, (b, lq, h, d)), (k_host, (b, lk, hkv, d)), (v_host, (b, lk, hkv, d)),
                        (out_host, (b, lq, h, d))):
            if tuple(t.shape) != want or not t.is_contiguous() or t.dtype != torch.bfloat16:
                raise ValueError(f"host tensor {tuple(t.shape)} is not a contiguous bf16 {want}")
        main = torch.cuda.current_stream(self.device)
        self.copy_in.wait_stream(main)   # the device buffers are free once earlier work is done
        self.copy_out.wait_stream(main)
        hg, kg = h // self.groups, hkv // self.groups
        loaded, done = [], []
        for g in range(self.groups):
            with torch.cuda.stream(self.copy_in):
                for dst, src in ((self.q, q_host), (self.k, k_host), (self.v, v_host)):
                    self._slice(dst, src, g, self.copy_in)
                ev = torch.cuda.Event()
                ev.record(self.copy_in)
                loaded.append(ev)
        for g in range(self.groups):
            main.wait_event(loaded[g])
            attention_fwd(self.q[:, :, g * hg:(g + 1) * hg], self.k[:, :, g * kg:(g + 1) * kg],
                          self.v[:, :, g * kg:(g + 1) * kg], out=self.out[:, :, g * hg:(g + 1) * hg],
                          return_lse=False)
            ev = torch.cuda.Event()
            ev.record(main)
            self.copy_out.wait_event(ev)
            self._slice(out_host, self.out, g, self.copy_out)
        fin = torch.cuda.Event()
        fin.record(self.copy_out)
        main.wait_event(fin)
        return out_host
