"""Ulysses sequence-parallel attention on NVLink peer windows.

One step, per rank (P ranks, local rows Ls = S/P, local heads Hl = H/P):
  1. dgxm_ulysses_scatter: this rank's (B, Ls, H, D) q/k/v rows are stored
     head-slice by head-slice straight into every peer's receive tensors
     (B, S, Hl, D) -- the rank-major gathered axis of yunchang's
     SeqAllToAll4D(pg, x, 2, 1) (adapters/usp_full_axis.py:27-29);
  2. dgxm_comm_barrier;
  3. dgxm_attn_fwd_routed: attention over the whole axis for the local heads,
     whose epilogue stores each output row into the (B, Ls, H, D) output of
     the rank owning that row -- the inverse SeqAllToAll4D(pg, out, 1, 2)
     (adapters/usp_full_axis.py:40) with no separate kernel;
  4. dgxm_comm_barrier.
At P = 1 the step is the attention kernel alone.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .comm import PeerWindows
from .ops import (_dtype_code, _ptr, _require_cuda, attention_fwd, attn_flags, kernel_head_dim,
                  out16_dtype)


def a2a_desc(n_tensors, world, rank, batch, seq_local, heads, head_dim, dtype, strides, seg0=0):
    d = _lib.A2ADesc()
    d.seg0 = int(seg0)
    d.n_tensors, d.world, d.rank = n_tensors, world, rank
    d.batch, d.seq_local, d.heads, d.head_dim = batch, seq_local, heads, head_dim
    d.dtype = _dtype_code(dtype)
    for t, st in enumerate(strides):
        d.src_stride[t][0], d.src_stride[t][1], d.src_stride[t][2] = st
    return d


def ulysses_scatter(tensors: list[torch.Tensor], dst_ptrs: list[list[int]], *, world: int,
                    rank: int, seg0: int = 0, stream=None) -> None:
    """Store head slices of this rank's (B, Ls, H, D) tensors into dst_ptrs[t][r].

    seg0 > 0 writes the joint (text-first canonical) order of a two-segment
    local layout instead of the rank-major concat.
    """
    _require_cuda(*tensors)
    b, ls, h, d = tensors[0].shape
    for t in tensors:
        if t.shape != tensors[0].shape or t.dtype != tensors[0].dtype or t.stride(3) != 1:
            raise ValueError("all-to-all tensors must share shape/dtype with contiguous head_dim")
    desc = a2a_desc(len(tensors), world, rank, b, ls, h, d, tensors[0].dtype,
                    [(t.stride(0), t.stride(1), t.stride(2)) for t in tensors], seg0)
    n = len(tensors)
    src = (ctypes.c_void_p * n)(*[t.data_ptr() for t in tensors])
    dst = (ctypes.c_void_p * (n * world))(*[p for row in dst_ptrs for p in row])
    stream = stream or torch.cuda.current_stream(tensors[0].device)
    _lib.check(_lib.load().dgxm_ulysses_scatter(ctypes.byref(desc), src, dst, stream.cuda_stream),
               "dgxm_ulysses_scatter")


def ulysses_scatter_copy(tensors: list[torch.Tensor], dst_ptrs: list[list[int]], *, world: int,
                         rank: int, stream=None) -> None:
    """The rank-major sequence->head scatter of ulysses_scatter as copy-engine
    transfers (dgxm_copy_2d): for each tensor and destination rank r, the head
    slice [r*H/P, (r+1)*H/P) of every local row is one strided copy into rows
    [rank*Ls, (rank+1)*Ls) of rank r's (B, P*Ls, H/P, D) receive tensor (one
    copy per batch item).  The same bytes as the kernel, but no SM is used, so
    it can run beside an attention launch without taking SM slots from it.
    Each row's heads must be contiguous (stride(2) == D)."""
    _require_cuda(*tensors)
    b, ls, h, d = tensors[0].shape
    if h % world:
        raise ValueError(f"{h} heads do not divide the Ulysses degree {world}")
    hl = h // world
    elt = tensors[0].element_size()
    for t in tensors:
        if t.shape != tensors[0].shape or t.dtype != tensors[0].dtype or t.stride(3) != 1 or t.stride(2) != d:
            raise ValueError("the copy-engine scatter needs (B, Ls, H, D) tensors with contiguous heads per row")
    from .ops import copy_2d

    stream = stream or torch.cuda.current_stream(tensors[0].device)
    row = hl * d * elt
    for t, dsts in zip(tensors, dst_ptrs):
        for r in range(world):
            for bi in range(b):
                src = t.data_ptr() + (bi * t.stride(0) + r * hl * d) * elt
                dst = dsts[r] + (bi * world * ls + rank * ls) * row
                copy_2d(dst, row, src, t.stride(1) * elt, row, ls, stream)


def ulysses_gather(src: torch.Tensor, dst_ptrs: list[int], *, world: int, rank: int,
                   seq_local: int, heads: int, seg0: int = 0, stream=None) -> None:
    """Return (B, S, Hl, D) rows to the owning ranks' (B, Ls, H, D) tensors."""
    _require_cuda(src)
    b, s, hl, d = src.shape
    if s != seq_local * world or hl * world != heads or src.stride(3) != 1:
        raise ValueError("gather source must be (B, world*seq_local, heads/world, D)")
    desc = a2a_desc(1, world, rank, b, seq_local, heads, d, src.dtype,
                    [(src.stride(0), src.stride(1), src.stride(2))], seg0)
    dst = (ctypes.c_void_p * world)(*dst_ptrs)
    stream = stream or torch.cuda.current_stream(src.device)
    _lib.check(_lib.load().dgxm_ulysses_gather(ctypes.byref(desc), src.data_ptr(), dst,
                                               stream.cuda_stream), "dgxm_ulysses_gather")


def attention_routed(q, k, v, out_ptrs: list[int], out_strides, *, world: int, rank: int,
                     seq_local: int, seg0: int = 0, lse: torch.Tensor | None = None,
                     softmax_scale=None,
                     q_descale=None, k_descale=None, v_descale=None, stream=None) -> None:
    """Attention whose epilogue writes row i to rank i // seq_local's output."""
    _require_cuda(q, k, v)
    b, lq, hl, d = q.shape
    _, lk, hkv, _ = k.shape
    desc = _lib.AttnDesc()
    desc.batch, desc.q_len, desc.kv_len = b, lq, lk
    desc.q_heads, desc.kv_heads, desc.head_dim = hl, hkv, d
    desc.in_dtype = _dtype_code(q.dtype)
    desc.out_dtype = _dtype_code(out16_dtype(q.dtype))
    desc.q_stride[:] = [q.stride(0), q.stride(1), q.stride(2)]
    desc.k_stride[:] = [k.stride(0), k.stride(1), k.stride(2)]
    desc.v_stride[:] = [v.stride(0), v.stride(1), v.stride(2)]
    desc.o_stride[:] = list(out_strides)
    if lse is not None:
        desc.lse_stride[:] = [lse.stride(0), lse.stride(1), lse.stride(2)]
    desc.softmax_scale = float(softmax_scale) if softmax_scale else 1.0 / math.sqrt(d)
    desc.flags = attn_flags()
    peers = (ctypes.c_void_p * world)(*out_ptrs)
    stream = stream or torch.cuda.current_stream(q.device)
    _lib.check(_lib.load().dgxm_attn_fwd_routed(
        ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(q_descale),
        _ptr(k_descale), _ptr(v_descale), peers, world, rank, seq_local, seg0, _ptr(lse),
        stream.cuda_stream), "dgxm_attn_fwd_routed")


class UlyssesAttention:
    """Ulysses-P attention for fixed (B, Ls, H, D) bf16 shapes on one rank."""

    def __init__(self, *, world: int, rank: int, batch: int, seq_local: int, heads: int,
                 head_dim: int, device: torch.device, group=None, generation: int = 0,
                 dtype: torch.dtype = torch.bfloat16) -> None:
        if heads % world:
            raise ValueError(f"{heads} heads do not divide the Ulysses degree {world}")
        self.world, self.rank, self.device = world, rank, device
        self.b, self.ls, self.h, self.d = batch, seq_local, heads, head_dim
        self.hl = heads // world
        self.s = seq_local * world
        self.dtype = dtype
        self.windows = None
        if world == 1:
            self.launches_per_step = 1
            return
        elt = torch.empty((), dtype=dtype).element_size()
        recv_bytes = batch * self.s * self.hl * head_dim * elt
        out_bytes = batch * seq_local * heads * head_dim * elt
        self.windows = PeerWindows(3 * recv_bytes + out_bytes + 4 * 256, device=device, group=group,
                                   rank=rank, world=world, generation=generation)
        self.off_recv = [self.windows.carve(recv_bytes) for _ in range(3)]
        self.off_out = self.windows.carve(out_bytes)
        self.recv = [self.windows.local_tensor(o, (batch, self.s, self.hl, head_dim), dtype)
                     for o in self.off_recv]
        self.out_local = self.windows.local_tensor(self.off_out, (batch, seq_local, heads, head_dim), dtype)
        self.out_strides = (seq_local * heads * head_dim, heads * head_dim, head_dim)
        self.lse = torch.empty(batch, self.hl, self.s, device=device, dtype=torch.float32)
        self.launches_per_step = 4

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        if self.world == 1:
            res, _ = attention_fwd(q, k, v, out=out, return_lse=False)
            return res
        w = self.windows
        ulysses_scatter([q, k, v], [[w.peer_ptr(r, off) for r in range(self.world)]
                                    for off in self.off_recv], world=self.world, rank=self.rank)
        w.barrier()
        attention_routed(self.recv[0], self.recv[1], self.recv[2],
                         [w.peer_ptr(r, self.off_out) for r in range(self.world)], self.out_strides,
                         world=self.world, rank=self.rank, seq_local=self.ls, lse=self.lse)
        w.barrier()
        if out is None:
            return self.out_local
        out.copy_(self.out_local)
        return out

    def time_attention_kernel(self, steps: int) -> float:
        """Mean ms of the attention kernel alone over this rank's full-axis heads."""
        if self.world == 1:
            g = torch.Generator(device=self.device).manual_seed(7)
            q, k, v = (torch.randn(self.b, self.s, self.h, self.d, device=self.device, generator=g,
                                   dtype=self.dtype) for _ in range(3))
        else:
            q, k, v = self.recv
        out = torch.empty(q.shape, device=self.device, dtype=self.dtype)
        for _ in range(2):
            attention_fwd(q, k, v, out=out, return_lse=False)
        stream = torch.cuda.current_stream(self.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            attention_fwd(q, k, v, out=out, return_lse=False)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    def close(self) -> None:
        if self.windows is not None:
            torch.cuda.synchronize(self.device)
            self.windows.close()
            self.windows = None


def ulysses_scatter_joint(tensors: list[torch.Tensor], texts: list[torch.Tensor] | None,
                          dst_ptrs: list[list[int]], *, world: int, rank: int,
                          text_first: bool = True, stream=None) -> None:
    """The scatter of joint attention with replicated text.

    tensors[t] is this rank's (B, Ls, H, D) image rows and texts[t] its whole
    (B, T, H, D) text (None: no text); dst_ptrs[t][r] is rank r's
    (B, T + world*Ls, H/world, D) receive tensor.  The image rows land
    rank-major after (text_first) or before the text rows; this rank's head
    slice of its own text goes into its own receive tensor only.
    """
    texts = list(texts or [])
    _require_cuda(*tensors, *texts)
    b, ls, h, d = tensors[0].shape
    for x in tensors:
        if x.shape != tensors[0].shape or x.dtype != tensors[0].dtype or x.stride(3) != 1:
            raise ValueError("image tensors must share shape/dtype with contiguous head_dim")
    tr = texts[0].shape[1] if texts else 0
    if texts and len(texts) != len(tensors):
        raise ValueError("one text tensor per image tensor")
    for x in texts:
        if (tuple(x.shape) != (b, tr, h, d) or x.dtype != tensors[0].dtype or x.stride(3) != 1):
            raise ValueError("text tensors must be (B, T, H, D) of the image dtype with contiguous head_dim")
    if tr == 0:
        texts = tensors  # never read: the library ignores text pointers without text rows
    desc = a2a_desc(len(tensors), world, rank, b, ls, h, d, tensors[0].dtype,
                    [(x.stride(0), x.stride(1), x.stride(2)) for x in tensors])
    n = len(tensors)
    src = (ctypes.c_void_p * n)(*[x.data_ptr() for x in tensors])
    txt = (ctypes.c_void_p * n)(*[x.data_ptr() for x in texts])
    strides = (ctypes.c_int64 * (3 * n))(*[s for x in texts for s in (x.stride(0), x.stride(1), x.stride(2))])
    dst = (ctypes.c_void_p * (n * world))(*[q for row in dst_ptrs for q in row])
    stream = stream or torch.cuda.current_stream(tensors[0].device)
    _lib.check(_lib.load().dgxm_ulysses_scatter_joint(ctypes.byref(desc), tr, 1 if text_first else 0, txt,
                                                      strides, src, dst, stream.cuda_stream),
               "dgxm_ulysses_scatter_joint")


class JointUlyssesAttention:
    """Ulysses joint image+text attention whose text every rank holds in full.

    The image rows are split by sequence over the P ranks and the text rows
    are replicated.  One step, per rank:
      1. dgxm_ulysses_scatter_joint: the image rows go head slice by head
         slice into every rank's receive tensors (rank-major), and this rank
         copies its head slice of its own text next to them -- no text
         crosses NVLink;
      2. dgxm_comm_barrier;
      3. attention over [text | image] ([image | text] when not text_first)
         for the local heads; the epilogue stores image rows to their owners
         and text rows to every rank at this rank's head columns, the
         all-gather of the text output over heads;
      4. dgxm_comm_barrier.
    The result is one-process attention over the unsharded concatenation:
    (image output (B, Ls, H, D) of this rank's rows, text output (B, T, H, D),
    the same on every rank).

    The step computes in `compute_dtype` (bf16, or fp16 for fp16 models):
    inputs of any float dtype are rounded to it and the outputs are returned
    in the inputs' own dtype, so an fp32 caller gets attention over its inputs
    rounded to bf16.  Head dimensions up to 64 run on the head-dim-64 kernel,
    larger ones below 128 (multiples of 8) zero-padded to 128: padded columns
    add exact zeros to every logit and give zero output columns, which are
    dropped; the softmax scale stays 1/sqrt(head_dim).
    """

    KERNEL_HEAD_DIM = 128

    def __init__(self, *, world: int, rank: int, batch: int, seq_local: int, txt_rows: int,
                 heads: int, head_dim: int, device: torch.device, text_first: bool = True,
                 group=None, generation: int = 0, softmax_scale: float | None = None,
                 compute_dtype: torch.dtype = torch.bfloat16) -> None:
        if compute_dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"joint attention computes in bf16 or fp16, not {compute_dtype}")
        if heads % world:
            raise ValueError(f"{heads} heads do not divide the Ulysses degree {world}")
        if head_dim > self.KERNEL_HEAD_DIM or head_dim % 8:
            raise ValueError(f"head_dim {head_dim} is not a multiple of 8 up to {self.KERNEL_HEAD_DIM}")
        if seq_local < 1 or txt_rows < 0:
            raise ValueError("each rank needs at least one image row and a non-negative text length")
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.world, self.rank, self.device = world, rank, device
        self.b, self.ls, self.t, self.h, self.d = batch, seq_local, txt_rows, heads, head_dim
        self.hl = heads // world
        self.text_first = text_first
        self.scale = softmax_scale or 1.0 / math.sqrt(head_dim)
        self.dk = dk = kernel_head_dim(head_dim)
        self.rows = txt_rows + world * seq_local
        self.dt = dt = compute_dtype
        recv_bytes = batch * self.rows * self.hl * dk * 2
        img_bytes = batch * seq_local * heads * dk * 2
        txt_bytes = batch * max(txt_rows, 1) * heads * dk * 2
        self.windows = PeerWindows(3 * recv_bytes + img_bytes + txt_bytes + 6 * 256, device=device,
                                   group=group, rank=rank, world=world, generation=generation)
        w = self.windows
        self.off_recv = [w.carve(recv_bytes) for _ in range(3)]
        self.off_img = w.carve(img_bytes)
        self.off_txt = w.carve(txt_bytes)
        self.recv = [w.local_tensor(o, (batch, self.rows, self.hl, dk), dt) for o in self.off_recv]
        self.img_out = w.local_tensor(self.off_img, (batch, seq_local, heads, dk), dt)
        self.txt_out = (w.local_tensor(self.off_txt, (batch, txt_rows, heads, dk), dt) if txt_rows > 0
                        else None)
        self.padded = head_dim != dk
        if self.padded:
            self.stage_img = [torch.zeros(batch, seq_local, heads, dk, device=device, dtype=dt) for _ in range(3)]
            self.stage_txt = [torch.zeros(batch, max(txt_rows, 1), heads, dk, device=device, dtype=dt)[:, :txt_rows]
                              for _ in range(3)]
        self.launches_per_step = 4 + (1 if txt_rows > 0 else 0)

    def _stage(self, xs, stage):
        if self.padded:
            for x, s in zip(xs, stage):
                s[..., :self.d].copy_(x)
            return stage
        return [x if x.device == self.device and x.dtype == self.dt and x.stride(3) == 1 else
                x.to(device=self.device, dtype=self.dt).contiguous() for x in xs]

    def forward(self, q_img, k_img, v_img, q_txt, k_txt, v_txt):
        for x in (q_img, k_img, v_img):
            if tuple(x.shape) != (self.b, self.ls, self.h, self.d):
                raise ValueError(f"image tensor {tuple(x.shape)} is not {(self.b, self.ls, self.h, self.d)}")
        for x in (q_txt, k_txt, v_txt):
            if tuple(x.shape) != (self.b, self.t, self.h, self.d):
                raise ValueError(f"text tensor {tuple(x.shape)} is not {(self.b, self.t, self.h, self.d)}")
        imgs = self._stage((q_img, k_img, v_img), self.stage_img if self.padded else None)
        txts = self._stage((q_txt, k_txt, v_txt), self.stage_txt if self.padded else None)
        w, p = self.windows, self.world
        ulysses_scatter_joint(list(imgs), list(txts) if self.t > 0 else None,
                              [[w.peer_ptr(r, off) for r in range(p)] for off in self.off_recv],
                              world=p, rank=self.rank, text_first=self.text_first)
        w.barrier()
        from .ops import attention_fwd_ext

        dk = self.dk
        route = {"o_peers": [w.peer_ptr(r, self.off_img) for r in range(p)], "world": p,
                 "rank": self.rank, "seq_local": self.ls,
                 "txt_rows": self.t, "txt_front": self.text_first,
                 "txt_peers": [w.peer_ptr(r, self.off_txt) for r in range(p)]}
        attention_fwd_ext(self.recv[0], self.recv[1], self.recv[2], route=route,
                          out_strides=(self.ls * self.h * dk, self.h * dk, dk),
                          softmax_scale=self.scale)
        w.barrier()
        img = self.img_out[..., :self.d].to(q_img.dtype, copy=True)
        if self.txt_out is None:
            return img, torch.empty(self.b, 0, self.h, self.d, device=self.device, dtype=q_img.dtype)
        return img, self.txt_out[..., :self.d].to(q_img.dtype, copy=True)

    __call__ = forward

    def close(self) -> None:
        if self.windows is not None:
            torch.cuda.synchronize(self.device)
            self.windows.close()
            self.windows = None


class HostStreamedUlysses:
    """Ulysses attention whose inputs and output live in pinned host memory,
    streamed one head group at a time.

    Each group of heads is a Ulysses step of its own (its heads divide the
    Ulysses degree), so the host->device copy of group g + 1 and the
    device->host copy of group g - 1 run on copy engines while group g is
    scattered, attended and gathered.  Each group's output is first copied out
    of the peer window on the compute stream, before any rank's next step can
    write into that window.
    """

    def __init__(self, *, world: int, rank: int, batch: int, seq_local: int, heads: int, head_dim: int,
                 device: torch.device, groups: int, group=None, generation: int = 0) -> None:
        if heads % groups or (heads // groups) % world:
            raise ValueError(f"{groups} head groups of {heads} heads do not split over {world} ranks")
        self.groups, self.device = groups, device
        self.shape = (batch, seq_local, heads, head_dim)
        self.uly = UlyssesAttention(world=world, rank=rank, batch=batch, seq_local=seq_local,
                                    heads=heads // groups, head_dim=head_dim, device=device, group=group,
                                    generation=generation)
        dt = torch.bfloat16
        self.q, self.k, self.v, self.out = (torch.empty(batch, seq_local, heads, head_dim, device=device, dtype=dt)
                                            for _ in range(4))
        self.copy_in = torch.cuda.Stream(device)
        self.copy_out = torch.cuda.Stream(device)
        self.launches_per_call = groups * self.uly.launches_per_step

    def __call__(self, q_host, k_host, v_host, out_host):
        from .ops import copy_2d

        b, ls, h, d = self.shape
        for t in (q_host, k_host, v_host, out_host):
            if tuple(t.shape) != self.shape or not t.is_contiguous() or t.dtype != torch.bfloat16:
                raise ValueError(f"host tensor {tuple(t.shape)} is not a contiguous bf16 {self.shape}")
        hg = h // self.groups
        pitch, width, rows = h * d * 2, hg * d * 2, b * ls
        main = torch.cuda.current_stream(self.device)
        self.copy_in.wait_stream(main)
        self.copy_out.wait_stream(main)
        loaded = []
        for g in range(self.groups):
            off = g * width
            for dst, src in ((self.q, q_host), (self.k, k_host), (self.v, v_host)):
                copy_2d(dst.data_ptr() + off, pitch, src.data_ptr() + off, pitch, width, rows, self.copy_in)
            ev = torch.cuda.Event()
            ev.record(self.copy_in)
            loaded.append(ev)
        for g in range(self.groups):
            sl = slice(g * hg, (g + 1) * hg)
            main.wait_event(loaded[g])
            self.uly.forward(self.q[:, :, sl], self.k[:, :, sl], self.v[:, :, sl], out=self.out[:, :, sl])
            ev = torch.cuda.Event()
            ev.record(main)
            self.copy_out.wait_event(ev)
            copy_2d(out_host.data_ptr() + g * width, pitch, self.out.data_ptr() + g * width, pitch, width, rows,
                    self.copy_out)
        fin = torch.cuda.Event()
        fin.record(self.copy_out)
        main.wait_event(fin)
        return out_host

    def close(self) -> None:
        self.uly.close()


class OverlappedUlysses:
    """A Ulysses step whose sequence->head scatter is hidden behind attention.

    The heads go in consecutive groups (each group's head count a multiple of
    the Ulysses degree): `groups` is a count of equal groups or a list of
    group sizes.  Group g + 1 is scattered on a side stream while the tensor
    cores attend group g; each group's routed epilogue writes its own head
    columns of the owners' outputs (the peer base pointers are offset by the
    group's first head), so the inverse all-to-all stays fused.  A small first
    group leaves only its own scatter exposed: at Ulysses-8 over 40 heads,
    [8, 32] exposes 8/40 of the all-to-all behind which one head per rank of
    attention hides the other 32.

    The first group's scatter, with nothing beside it, runs the SM kernel; the
    later ones run on copy engines (ulysses_scatter_copy), so they take no SM
    from the attention launch they run beside.

    Receive slots: two groups use one slot each.  With more groups two slots
    alternate, and a rank refills a slot in its peers' windows only after a
    barrier that every rank reaches after its own attention from that slot, so
    no peer still reads it.  All barriers of the windows are ordered through
    the two streams' events, as their shared epoch counter requires.  The
    result is bit-identical to UlyssesAttention.forward.
    """

    def __init__(self, *, world: int, rank: int, batch: int, seq_local: int, heads: int, head_dim: int,
                 device: torch.device, groups, group=None, generation: int = 0,
                 dtype: torch.dtype = torch.bfloat16) -> None:
        if world < 2:
            raise ValueError("the overlapped step needs a Ulysses degree of 2 or more")
        if isinstance(groups, int):
            if groups < 1 or heads % groups:
                raise ValueError(f"{groups} groups do not split {heads} heads evenly")
            sizes = [heads // groups] * groups
        else:
            sizes = [int(n) for n in groups]
        if sum(sizes) != heads or any(n < 1 or n % world for n in sizes):
            raise ValueError(f"head groups {sizes} do not split {heads} heads into multiples of {world} ranks")
        self.world, self.rank, self.device = world, rank, device
        self.sizes = sizes
        self.groups = len(sizes)
        self.first = [sum(sizes[:g]) for g in range(self.groups)]   # first head of each group
        self.b, self.ls, self.h, self.d = batch, seq_local, heads, head_dim
        s = seq_local * world
        elt = torch.empty((), dtype=dtype).element_size()
        self.n_slots = min(2, self.groups)
        # slot i serves groups i, i + 2, ...: sized for the largest of them
        slot_heads = [max(sizes[i::2]) // world for i in range(self.n_slots)]
        slot_bytes = [batch * s * hl * head_dim * elt for hl in slot_heads]
        out_bytes = batch * seq_local * heads * head_dim * elt
        self.windows = PeerWindows(3 * sum(slot_bytes) + out_bytes + 8 * 256, device=device, group=group,
                                   rank=rank, world=world, generation=generation)
        self.off_recv = [[self.windows.carve(nb) for _ in range(3)] for nb in slot_bytes]
        self.off_out = self.windows.carve(out_bytes)
        self.s, self.dtype = s, dtype
        self.out_local = self.windows.local_tensor(self.off_out, (batch, seq_local, heads, head_dim), dtype)
        self.out_strides = (seq_local * heads * head_dim, heads * head_dim, head_dim)
        self.head_bytes = head_dim * elt
        self.side = torch.cuda.Stream(device)
        # per group a scatter, a barrier and an attention; a slot-reuse barrier
        # per group after the first two; the final barrier
        self.launches_per_step = 3 * self.groups + max(0, self.groups - 2) + 1

    def _recv(self, g: int):
        hl = self.sizes[g] // self.world
        return [self.windows.local_tensor(off, (self.b, self.s, hl, self.d), self.dtype)
                for off in self.off_recv[g % 2]]

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        w, side = self.windows, self.side
        main = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(main)
        side.wait_event(start)       # inputs written, the previous step finished
        ready: list = [None] * self.groups
        freed: list = [None, None]

        def scatter(g: int) -> None:
            slot = g % 2
            if g >= 2:
                side.wait_event(freed[slot])   # this rank attended group g - 2 from the slot
                w.barrier(side)                 # ... and so has every other rank
            sl = slice(self.first[g], self.first[g] + self.sizes[g])
            xs = [q[:, :, sl], k[:, :, sl], v[:, :, sl]]
            dst = [[w.peer_ptr(r, off) for r in range(self.world)] for off in self.off_recv[slot]]
            if g == 0:
                # Nothing runs beside the first group's scatter, so the SM
                # kernel moves it: copy engines take one strided copy per
                # peer and tensor, slow for its one-head rows.
                ulysses_scatter(xs, dst, world=self.world, rank=self.rank, stream=side)
            else:
                # Copy engines move the group beside the attention of the
                # group before it, taking no SM from that launch.
                ulysses_scatter_copy(xs, dst, world=self.world, rank=self.rank, stream=side)
            w.barrier(side)                     # every rank's rows of group g have landed
            ev = torch.cuda.Event()
            ev.record(side)
            ready[g] = ev

        for g in range(min(2, self.groups)):
            scatter(g)
        for g in range(self.groups):
            main.wait_event(ready[g])
            qg, kg, vg = self._recv(g)
            col = self.first[g] * self.head_bytes
            attention_routed(qg, kg, vg, [w.peer_ptr(r, self.off_out) + col for r in range(self.world)],
                             self.out_strides, world=self.world, rank=self.rank, seq_local=self.ls)
            ev = torch.cuda.Event()
            ev.record(main)
            freed[g % 2] = ev
            if g + 2 < self.groups:
                scatter(g + 2)
        w.barrier(main)                         # every routed row of every group has landed
        if out is None:
            return self.out_local
        out.copy_(self.out_local)
        return out

    def close(self) -> None:
        if self.windows is not None:
            torch.cuda.synchronize(self.device)
            self.windows.close()
            self.windows = None
