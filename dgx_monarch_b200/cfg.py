"""CFG-parallel: cond/uncond batch rows across the ranks of a cfg group.

The reference splits one batched cond+uncond model call into
`batch // world` contiguous rows per cfg rank, runs the forward, and
all-gathers the predictions over the cfg group
(adapters/cfg_parallel.py:57-87 slicing, :293-301 gather, :304-374 the
wrapper).  Here the slice follows the same contract and the gather is a
peer-store all-gather into NVLink windows (dgxm_comm_allgather): each rank's
prediction is copied straight into every peer's window, then a bounded flag
barrier, with no NCCL call on the data path.  CFG pairs map to GPU pairs: with
sequence parallel fastest, rank r and r + sp form a pair (cfg_rank_layout).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .comm import PeerWindows
from .ops import _require_cuda, _require_on


class UnsupportedModelError(RuntimeError):
    """Typed refusal (adapters/base.py:37)."""


def _children(item) -> list:
    """The direct members of a forward argument container (dict values in
    insertion order, list / tuple items); leaves have none."""
    if isinstance(item, dict):
        return list(item.values())
    if isinstance(item, (list, tuple)):
        return list(item)
    return []


def _rebuild(item, fn):
    """`item` with `fn` applied to every leaf, containers rebuilt as the same
    kind (a tuple stays a tuple, a dict keeps its keys)."""
    if isinstance(item, dict):
        return {key: _rebuild(member, fn) for key, member in item.items()}
    if isinstance(item, tuple):
        return tuple(_rebuild(member, fn) for member in item)
    if isinstance(item, list):
        return [_rebuild(member, fn) for member in item]
    return fn(item)


def take_slice(value, batch: int, world: int, rank: int):
    """The cfg rank's share of one batched model call
    (adapters/cfg_parallel.py:71-87): a tensor whose leading dimension is the
    whole call batch keeps rows [rank * n, (rank + 1) * n), n = batch // world,
    as a view; every other leaf (broadcast tensors, scalars, non-tensors)
    is shared unchanged, and containers are rebuilt around their members."""
    share = batch // world
    first = rank * share

    def rows_of(leaf):
        if torch.is_tensor(leaf) and leaf.dim() > 0 and leaf.size(0) == batch:
            return leaf[first:first + share]
        return leaf

    return _rebuild(value, rows_of)


def leading_batch(value) -> int | None:
    """Leading dimension of the first tensor found in a forward argument,
    searching containers level by level (adapters/cfg_parallel.py:57-68);
    None when that tensor is a scalar or there is no tensor."""
    level = [value]
    while level:
        for item in level:
            if torch.is_tensor(item):
                return int(item.size(0)) if item.dim() > 0 else None
        level = [member for item in level for member in _children(item)]
    return None


def cfg_rank_layout(world: int, sp: int, cfg: int) -> list[tuple[int, int]]:
    """(sp_rank, cfg_rank) per global rank: sequence parallel fastest, then cfg."""
    if world % (sp * cfg):
        raise ValueError(f"world {world} is not a multiple of sp*cfg={sp * cfg}")
    return [(r % sp, (r // sp) % cfg) for r in range(world)]


class CfgGather:
    """Peer-store all-gather of fixed-size predictions over one cfg group.

    Two window buffers alternate by call: a rank copies into buffer
    (n+1) % 2 only after passing the barrier of call n, which every peer
    reaches after reading its call n-1 result out of that buffer."""

    def __init__(self, nbytes_per_rank: int, *, device: torch.device, group=None, rank: int = 0,
                 world: int = 1, generation: int = 0) -> None:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            # The named group, or the default group when none is given.
            rank, world = dist.get_rank(group), dist.get_world_size(group)
        span = (nbytes_per_rank * max(world, 1) + 255) // 256 * 256
        self.windows = PeerWindows(2 * span + 256, device=device, group=group, rank=rank, world=world,
                                   generation=generation)
        self.world, self.rank, self.device = self.windows.world, self.windows.rank, device
        self.slice_bytes = nbytes_per_rank
        self.offsets = (self.windows.carve(span), self.windows.carve(span))
        self.calls = 0

    def gather_in_window(self, local: torch.Tensor) -> torch.Tensor:
        """Gather into this call's window buffer and return a view of it, valid
        until the call after next."""
        _require_on(self.device, local)
        local = local.contiguous()
        nbytes = local.numel() * local.element_size()
        if nbytes != self.slice_bytes:
            raise ValueError(f"gather planned for {self.slice_bytes} bytes per rank, got {nbytes}")
        offset = self.offsets[self.calls % 2]
        self.calls += 1
        stream = torch.cuda.current_stream(self.device)
        _lib.check(_lib.load().dgxm_comm_allgather(self.windows._handle, local.data_ptr(), nbytes,
                                                    offset, stream.cuda_stream),
                   "dgxm_comm_allgather")
        return self.windows.local_tensor(offset, (self.world * local.shape[0], *local.shape[1:]),
                                         local.dtype)

    def __call__(self, local: torch.Tensor) -> torch.Tensor:
        return self.gather_in_window(local).clone()

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        self.windows.close()


_PRED_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16,
                torch.float16: _lib.DTYPE_F16}


def cfg_combine(cond: torch.Tensor, uncond: torch.Tensor, cfg: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """uncond + (cond - uncond) * cfg, rounded per operation as torch does
    (comfy's default cfg_function), in one kernel (dgxm_cfg_combine)."""
    if cond.shape != uncond.shape or cond.dtype != uncond.dtype or cond.dtype not in _PRED_DTYPES:
        raise ValueError("cond and uncond must share shape and a float dtype")
    _require_cuda(cond, uncond, out)
    if out is not None and (out.shape != cond.shape or out.dtype != cond.dtype or not out.is_contiguous()
                            or out.data_ptr() % 16):
        raise ValueError("out must be a contiguous, 16-byte aligned tensor of the predictions' shape and dtype")
    # The kernel moves 16-byte vectors; a view at an unaligned offset (a
    # prediction whose byte size is not a multiple of 16, sliced out of the
    # gathered pair) is copied to an aligned buffer first.
    cond, uncond = (t.contiguous() if t.data_ptr() % 16 == 0 else t.clone() for t in (cond, uncond))
    if out is None:
        out = torch.empty_like(cond)
    stream = torch.cuda.current_stream(cond.device)
    _lib.check(_lib.load().dgxm_cfg_combine(cond.data_ptr(), uncond.data_ptr(), cond.numel(),
                                            _PRED_DTYPES[cond.dtype], float(cfg), out.data_ptr(),
                                            stream.cuda_stream), "dgxm_cfg_combine")
    return out


class DualModelCfg:
    """The dm-cfg2 exchange (actor/dual_model_cfg.py:75-94): cfg rank 0 runs
    the conditional model, rank 1 the unconditional one; each step both
    predictions cross NVLink into both ranks' windows (cond first, the
    all-gather's rank order) and both ranks combine them with the same
    fp32 formula, so the samplers evolve identically."""

    def __init__(self, pred_bytes: int, cfg: float, *, device: torch.device, group=None,
                 generation: int = 0) -> None:
        import math

        if math.isclose(float(cfg), 1.0):
            # actor/dual_model_cfg.py:122-130: at cfg 1.0 the unconditional
            # rank would have no work and skip the exchange its peer waits in.
            raise UnsupportedModelError(
                "dual-model cfg-parallel (cfg2) needs a guider cfg above 1: at cfg 1.0 the "
                "unconditional rank has no guidance work and would skip the per-step exchange, "
                "hanging its peer. Raise the guider cfg above 1, or run this render at cfg 1.0 "
                "on topology uly2 instead.")
        self.cfg = float(cfg)
        self.gather = CfgGather(pred_bytes, device=device, group=group, generation=generation)
        if self.gather.world != 2:
            raise UnsupportedModelError(
                f"dual-model cfg splits across a cfg group of 2 ranks, not {self.gather.world}")

    def __call__(self, local_pred: torch.Tensor) -> torch.Tensor:
        both = self.gather.gather_in_window(local_pred)
        n = local_pred.shape[0]
        return cfg_combine(both[:n], both[n:2 * n], self.cfg)

    def close(self) -> None:
        self.gather.close()


def cfg_parallel_call(forward, *args, batch_arg: str = "x", group=None, gather: CfgGather | None = None,
                      **kwargs):
    """Run `forward` on this cfg rank's rows and gather the full prediction.

    Mirrors the reference wrapper's contract (adapters/cfg_parallel.py:
    343-372): the batch comes from `batch_arg`, must split into equal
    slices, every tensor argument with that leading size is sliced, and the
    result is all-gathered in rank order.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    if world <= 1:
        return forward(*args, **kwargs)
    x = kwargs.get(batch_arg, args[0] if args else None)
    batch = leading_batch(x)
    if batch is None or batch < world or batch % world:
        raise UnsupportedModelError(
            f"cfg-parallel got a model call of batch={batch}, which does not split into {world} "
            "equal slices.")
    sl_args = [take_slice(a, batch, world, rank) for a in args]
    sl_kwargs = {k: take_slice(v, batch, world, rank) for k, v in kwargs.items()}
    local = forward(*sl_args, **sl_kwargs)
    if gather is None:
        raise ValueError("cfg_parallel_call needs a CfgGather sized for the prediction slice")
    return gather(local)
