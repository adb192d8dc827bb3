"""Sequence shards: pad / chunk, the NVLink all-gather behind sp_gather, and
the shared NVFP4 activation scale.

- `pad_seq_to_multiple` and `shard_seq` give the zero pad and the per-rank
  chunk of adapters/base.py:48-123 (a view of the stream where the chunk
  lies inside it; only a chunk reaching into the pad is assembled).
- `SequenceGather` replaces `sp_gather` (adapters/base.py:126-131), the
  xfuser all-gather of every rank's chunk followed by a trim to the declared
  length: each rank peer-stores its rows into every rank's window in the
  trimmed layout (libdgxm_sp.so: dgxm_seq_allgather).
- `SharedActivationScale` replaces the max all-reduce of
  `shared_activation_scale` (adapters/quant_activation_scale.py:222-246):
  local amax, exchange and reduce over the peer windows, then
  `dtype(amax) / divisor` in the activation dtype
  (dgxm_shared_amax_scale).

Every rank of the group calls these in the same order with the same shapes,
as the reference's collectives require.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .comm import PeerWindows
from .ops import _require_on

NVFP4_SCALE_DIVISOR = 448.0 * 6.0  # F8_E4M3_MAX * F4_E2M1_MAX (adapters/quant_activation_scale.py:91-100)


_ACT_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16,
               torch.float32: _lib.DTYPE_F32}


class ShardRefusal(RuntimeError):
    """Typed refusal of shard_seq(allow_padding=False) on an indivisible stream."""


def pad_seq_to_multiple(t: torch.Tensor, multiple: int, dim: int = 1) -> tuple[torch.Tensor, int]:
    """`t` with zero rows appended along `dim` up to the next multiple of
    `multiple` (the tensor itself when none are needed), and its original
    length -- the divisibility pad of adapters/base.py:48-56."""
    length = t.size(dim)
    target = -(-length // multiple) * multiple
    if target == length:
        return t, length
    shape = list(t.shape)
    shape[dim] = target
    padded = t.new_zeros(shape)
    padded.narrow(dim, 0, length).copy_(t)
    return padded, length


def shard_seq(t: torch.Tensor | None, world: int, rank: int, dim: int = 1, *,
              allow_padding: bool = True, name: str | None = None):
    """This rank's contiguous chunk of the zero-padded stream and the stream's
    length before the pad (the contract of adapters/base.py:91-123).

    The padded stream is never built: a chunk that lies inside the stream is
    a view of it, and only a chunk that reaches past the end is assembled,
    from its real rows and zeros."""
    if t is None:
        return None, 0
    length = t.size(dim)
    if length % world and not allow_padding:
        subject = f"{name} stream" if name else "sequence"
        raise ShardRefusal(
            f"{subject} length {length} on dim {dim} is not divisible by the sequence-parallel "
            f"degree {world}, and this adapter requires exact divisibility.")
    step = -(-length // world)
    start = rank * step
    if start + step <= length:
        return t.narrow(dim, start, step), length
    shape = list(t.shape)
    shape[dim] = step
    chunk = t.new_zeros(shape)
    real = max(0, length - start)
    if real:
        chunk.narrow(dim, 0, real).copy_(t.narrow(dim, start, real))
    return chunk, length


def _rank_world(group) -> tuple[int, int]:
    """This process's rank and the size of `group` (the default group when
    None), or (0, 1) without torch.distributed."""
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def _new_windows(nbytes: int, device, group, generation) -> PeerWindows:
    rank, world = _rank_world(group)
    return PeerWindows(nbytes, device=device, group=group, rank=rank, world=world, generation=generation)


def _windows_for(cache: dict, nbytes: int, device, group, generation) -> PeerWindows:
    """A window at least `nbytes` large; grows by replacing (collective)."""
    win = cache.get("win")
    if win is None or win.nbytes < nbytes:
        if win is not None:
            torch.cuda.synchronize(device)
            win.close()
        win = _new_windows(max(nbytes, 1 << 20), device, group, generation)
        cache["win"] = win
    return win


def seq_gather_store(src: torch.Tensor, orig_len: int, dst_ptrs: list[int], *, world: int,
                     rank: int, stream=None) -> None:
    """The store half of sp_gather (dgxm_seq_gather_store): this rank's rows of
    a contiguous (B, L, row) tensor whose rows are whole 16-byte units go into
    rank r's trimmed (B, orig_len, row) buffer at dst_ptrs[r], gathered rows
    [rank * L, (rank + 1) * L) below orig_len; no barrier."""
    _require_on(src.device, src)
    if src.ndim != 3 or not src.is_contiguous():
        raise ValueError("the gather source is a contiguous (B, L, row) tensor")
    if len(dst_ptrs) != world:
        raise ValueError(f"{len(dst_ptrs)} destinations for {world} ranks")
    b, seq_local, row = src.shape
    row_bytes = row * src.element_size()
    desc = _lib.SeqGatherDesc()
    desc.batch, desc.seq_local, desc.orig_len, desc.row_bytes = b, seq_local, orig_len, row_bytes
    desc.src_batch_stride = seq_local * row_bytes
    desc.src_row_stride = row_bytes
    dst = (ctypes.c_void_p * world)(*dst_ptrs)
    stream = stream or torch.cuda.current_stream(src.device)
    _lib.check(_lib.load().dgxm_seq_gather_store(ctypes.byref(desc), world, rank, src.data_ptr(), dst,
                                                 stream.cuda_stream), "dgxm_seq_gather_store")


class SequenceGather:
    """`sp_gather(t, orig_len, dim)` over NVLink for one sequence group.

    Two window buffers alternate by call: a rank writes buffer (n+1) % 2 only
    after passing the barrier of call n, which each peer reaches after copying
    out its call n-1 result from that buffer, in stream order."""

    def __init__(self, *, group=None, device: torch.device | None = None, generation: int = 0) -> None:
        self.group, self.generation = group, generation
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self._cache: dict = {}
        self._calls = 0
        self.closed = False

    def __call__(self, t: torch.Tensor, orig_len: int, dim: int = 1) -> torch.Tensor:
        if self.closed:
            raise RuntimeError("this sequence gather belongs to a retired setup generation")
        _require_on(self.device, t)
        dim = dim % t.ndim
        t = t.contiguous()
        lead = math.prod(t.shape[:dim])
        seq_local = t.shape[dim]
        row_elems = math.prod(t.shape[dim + 1:])
        elt = t.element_size()
        row_bytes = row_elems * elt
        send_row = (row_bytes + 15) // 16 * 16  # the kernel moves 16-byte units
        buf = (lead * orig_len * send_row + 255) // 256 * 256
        win = _windows_for(self._cache, 2 * buf, self.device, self.group, self.generation)
        if orig_len > seq_local * win.world or orig_len < 0:
            raise ValueError(f"orig_len {orig_len} exceeds {win.world} x {seq_local} gathered rows")
        src = t.reshape(lead, seq_local, row_elems)
        if send_row != row_bytes:
            src = torch.nn.functional.pad(src, (0, (send_row - row_bytes) // elt))
        offset = (self._calls % 2) * buf
        self._calls += 1
        desc = _lib.SeqGatherDesc()
        desc.batch, desc.seq_local, desc.orig_len, desc.row_bytes = lead, seq_local, orig_len, send_row
        desc.src_batch_stride = seq_local * send_row
        desc.src_row_stride = send_row
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.load().dgxm_seq_allgather(win._handle, ctypes.byref(desc), src.data_ptr(), offset,
                                                  stream), "dgxm_seq_allgather")
        got = win.local_tensor(offset, (lead, orig_len, send_row // elt), t.dtype)[..., :row_elems]
        return got.reshape(*t.shape[:dim], orig_len, *t.shape[dim + 1:]).clone()

    def close(self) -> None:
        win = self._cache.pop("win", None)
        if win is not None:
            torch.cuda.synchronize(self.device)
            win.close()
        self.closed = True


class SharedActivationScale:
    """The NVFP4 activation scale a single GPU would take over the whole tensor,
    for the ranks of `group` (the sequence x CFG ranks of one model call)."""

    def __init__(self, *, group=None, device: torch.device | None = None, generation: int = 0) -> None:
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.windows = _new_windows(1 << 16, self.device, group, generation)

    def __call__(self, input: torch.Tensor, divisor: float = NVFP4_SCALE_DIVISOR,
                 trace: list | None = None) -> torch.Tensor:
        """0-d scale in input's dtype: dtype(max over ranks of amax|x|) / divisor."""
        if input.dtype not in _ACT_DTYPES:
            raise ValueError(f"activation dtype {input.dtype} has no NVFP4 activation scale")
        _require_on(self.device, input)
        flat = input.reshape(-1, input.shape[-1]) if input.ndim >= 1 and input.numel() else input.reshape(0, 1)
        if flat.stride(-1) != 1:
            flat = flat.contiguous()
        scale = torch.empty((), device=self.device, dtype=input.dtype)
        amax = torch.empty(1, device=self.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.load().dgxm_shared_amax_scale(
            self.windows._handle, flat.data_ptr() if flat.numel() else None, flat.shape[0], flat.shape[1],
            flat.stride(0), _ACT_DTYPES[input.dtype], float(divisor), scale.data_ptr(), amax.data_ptr(),
            stream), "dgxm_shared_amax_scale")
        if trace is not None:
            local = (torch.zeros(1, device=self.device, dtype=torch.float32) if flat.numel() == 0
                     else flat.abs().amax().to(torch.float32).reshape(1))
            trace.extend((local, amax))
        return scale

    def close(self) -> None:
        if self.windows is not None:
            torch.cuda.synchronize(self.device)
            self.windows.close()
            self.windows = None
