"""Ring attention over one ring group (libdgxm_sp.so: dgxm_ring_attn_fwd).

Each rank holds its query rows and one key/value block of the sequence.  The
blocks rotate over NVLink into the next rank's peer window (copy engines,
overlapped with attention on the current block) and the per-block results
merge by log-sum-exp in fp32.  This replaces the ring loop the reference
reaches through xfuser/yunchang (adapters/base.py:320 with ring degree > 1);
the rotation order matches oracle.usp.ring_attention (rank r attends the block
of rank (r - t) mod R at step t).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .comm import PeerWindows
from .ops import _ptr, _require_on, attn_desc, check_attn_buffers, out16_dtype


class RingAttention:
    """Ring attention for fixed shapes on one rank of a ring group."""

    def __init__(self, *, world: int, rank: int, batch: int, q_len: int, kv_len: int, heads: int,
                 kv_heads: int, head_dim: int, device: torch.device, group=None,
                 generation: int = 0, dtype: torch.dtype = torch.bfloat16,
                 timeout_ms: int | None = None) -> None:
        self.world, self.rank, self.device = world, rank, device
        self.shape = (batch, q_len, kv_len, heads, kv_heads, head_dim)
        probe_q = torch.empty(batch, q_len, heads, head_dim, device="meta", dtype=dtype)
        probe_k = torch.empty(batch, kv_len, kv_heads, head_dim, device="meta", dtype=dtype)
        desc = attn_desc(probe_q, probe_k, probe_k, probe_q, None)
        lib = _lib.load()
        self.window_bytes = int(lib.dgxm_ring_window_bytes(ctypes.byref(desc)))
        self.workspace_bytes = int(lib.dgxm_ring_workspace_bytes(ctypes.byref(desc), world))
        self.windows = PeerWindows(self.window_bytes, device=device, group=group, rank=rank,
                                   world=world, generation=generation)
        if timeout_ms is not None:
            _lib.check(lib.dgxm_comm_set_timeout(self.windows._handle, int(timeout_ms)),
                       "dgxm_comm_set_timeout")
        self.workspace = torch.empty(self.workspace_bytes, dtype=torch.uint8, device=device)
        self.launches_per_step = 2 * world  # attention per block, barriers, merge

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
                softmax_scale: float | None = None, q_descale: torch.Tensor | None = None,
                k_descale: torch.Tensor | None = None,
                v_descale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
        """e4m3 inputs (a ring planned with dtype float8_e4m3fn) take per-head
        fp32 descales: q's for the local rows, k's and v's for this rank's
        block; the output is bf16."""
        b, lq, h, d = q.shape
        if (b, lq, k.shape[1], h, k.shape[2], d) != self.shape or v.shape != k.shape:
            raise ValueError(f"ring planned for {self.shape}, called with q {tuple(q.shape)} k {tuple(k.shape)}")
        _require_on(self.device, q, k, v, q_descale, k_descale, v_descale)
        check_attn_buffers(q, k, out=out, lse=lse, q_descale=q_descale, k_descale=k_descale,
                           v_descale=v_descale)
        k, v = k.contiguous(), v.contiguous()
        if out is None:
            out = torch.empty(b, lq, h, d, device=self.device, dtype=out16_dtype(q.dtype))
        desc = attn_desc(q, k, v, out, lse, softmax_scale)
        stream = torch.cuda.current_stream(self.device)
        lib = _lib.load()
        if q.dtype == torch.float8_e4m3fn:
            _lib.check(lib.dgxm_ring_attn_fwd_fp8(
                self.windows._handle, ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                _ptr(q_descale), _ptr(k_descale), _ptr(v_descale), out.data_ptr(), _ptr(lse),
                self.workspace.data_ptr(), self.workspace_bytes, stream.cuda_stream),
                "dgxm_ring_attn_fwd_fp8")
        else:
            _lib.check(lib.dgxm_ring_attn_fwd(
                self.windows._handle, ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                out.data_ptr(), _ptr(lse), self.workspace.data_ptr(), self.workspace_bytes,
                stream.cuda_stream), "dgxm_ring_attn_fwd")
        return out, lse

    def close(self) -> None:
        if self.windows is not None:
            torch.cuda.synchronize(self.device)
            self.windows.close()
            self.windows = None


def kv_gather_store(k: torch.Tensor, v: torch.Tensor, dst_k: list[int], dst_v: list[int], *,
                    world: int, rank: int, stream=None) -> None:
    """The store half of the full-context gather (dgxm_kv_gather_store): this
    rank's (B, L, H_kv, 128) K and V blocks (16-bit, any 16-byte strides) go
    into rows [rank * L, (rank + 1) * L) of every rank's contiguous
    (B, world * L, H_kv, 128) full K / V at dst_k[r] / dst_v[r]; no barrier."""
    _require_on(k.device, k, v)
    if k.shape != v.shape or k.dtype != v.dtype or k.ndim != 4:
        raise ValueError("k and v are equal (B, L, H_kv, D) blocks of one dtype")
    if len(dst_k) != world or len(dst_v) != world:
        raise ValueError(f"destinations for {world} ranks expected")
    desc = attn_desc(k, k, v, k, None)
    stream = stream or torch.cuda.current_stream(k.device)
    _lib.check(_lib.load().dgxm_kv_gather_store(
        ctypes.byref(desc), world, rank, k.data_ptr(), v.data_ptr(), (ctypes.c_void_p * world)(*dst_k),
        (ctypes.c_void_p * world)(*dst_v), stream.cuda_stream), "dgxm_kv_gather_store")


class FullContextRingAttention:
    """Local Q against the whole K/V axis of a ring group, in one kernel call
    (libdgxm_sp.so: dgxm_full_context_attn_fwd).

    The Wan Ring2 full-context path of the reference
    (adapters/wan_ring_full_context.py:203-295, :422-449): each rank's K/V
    block lands in rank-major slots of every rank's peer window (NVLink peer
    stores, all batch items at once), then one attention call of the local
    query rows over the gathered axis -- exact, with no LSE merge.
    """

    def __init__(self, *, world: int, rank: int, batch: int, q_len: int, kv_len: int, heads: int,
                 kv_heads: int, head_dim: int, device: torch.device, group=None,
                 generation: int = 0, timeout_ms: int | None = None,
                 dtype: torch.dtype = torch.bfloat16) -> None:
        self.world, self.rank, self.device = world, rank, device
        self.shape = (batch, q_len, kv_len, heads, kv_heads, head_dim)
        probe_q = torch.empty(batch, q_len, heads, head_dim, device="meta", dtype=dtype)
        probe_k = torch.empty(batch, kv_len, kv_heads, head_dim, device="meta", dtype=dtype)
        desc = attn_desc(probe_q, probe_k, probe_k, probe_q, None)
        lib = _lib.load()
        self.window_bytes = int(lib.dgxm_full_context_window_bytes(ctypes.byref(desc), world))
        self.windows = PeerWindows(self.window_bytes, device=device, group=group, rank=rank,
                                   world=world, generation=generation)
        if timeout_ms is not None:
            _lib.check(lib.dgxm_comm_set_timeout(self.windows._handle, int(timeout_ms)),
                       "dgxm_comm_set_timeout")
        self.launches_per_step = 3  # gather, barrier, attention

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
                softmax_scale: float | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
        b, lq, h, d = q.shape
        if (b, lq, k.shape[1], h, k.shape[2], d) != self.shape or v.shape != k.shape:
            raise ValueError(f"full-context ring planned for {self.shape}, called with "
                             f"q {tuple(q.shape)} k {tuple(k.shape)} v {tuple(v.shape)}")
        _require_on(self.device, q, k, v)
        check_attn_buffers(q, k, out=out, lse=lse)
        if out is None:
            out = torch.empty(b, lq, h, d, device=self.device, dtype=q.dtype)
        desc = attn_desc(q, k, v, out, lse, softmax_scale)
        stream = torch.cuda.current_stream(self.device)
        _lib.check(_lib.load().dgxm_full_context_attn_fwd(
            self.windows._handle, ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(),
            out.data_ptr(), _ptr(lse), stream.cuda_stream), "dgxm_full_context_attn_fwd")
        return out, lse

    def close(self) -> None:
        if self.windows is not None:
            torch.cuda.synchronize(self.device)
            self.windows.close()
            self.windows = None
