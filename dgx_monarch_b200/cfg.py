"""CFG-parallel: cond/uncond batch rows across the ranks of a cfg group.

The reference splits one batched cond+uncond model call into
`batch // world` contiguous rows per cfg rank, runs the forward, and
all-gathers the predictions over the cfg group
(adapters/cfg_parallel.py:57-87 slicing, :293-301 gather, :304-374 the
wrapper).  Here the slicing mirrors `_take_slice` exactly and the gather is a
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


class UnsupportedModelError(RuntimeError):
    """Typed refusal (adapters/base.py:37)."""


def take_slice(value, batch: int, world: int, rank: int):
    """This rank's contiguous rows of every tensor whose dim 0 equals the call
    batch; broadcast tensors and non-tensor leaves pass through; containers
    recurse (adapters/cfg_parallel.py:71-87)."""
    if torch.is_tensor(value):
        if value.ndim > 0 and value.shape[0] == batch:
            rows = batch // world
            return value.narrow(0, rank * rows, rows)
        return value
    if isinstance(value, dict):
        return {key: take_slice(item, batch, world, rank) for key, item in value.items()}
    if isinstance(value, (list, tuple)):
        sliced = [take_slice(item, batch, world, rank) for item in value]
        return tuple(sliced) if isinstance(value, tuple) else sliced
    return value


def leading_batch(value) -> int | None:
    """Batch size of the first tensor inside a forward argument
    (adapters/cfg_parallel.py:57-68)."""
    queue = [value]
    while queue:
        item = queue.pop(0)
        if torch.is_tensor(item):
            return int(item.shape[0]) if item.ndim > 0 else None
        if isinstance(item, dict):
            queue.extend(item.values())
        elif isinstance(item, (list, tuple)):
            queue.extend(item)
    return None


def cfg_rank_layout(world: int, sp: int, cfg: int) -> list[tuple[int, int]]:
    """(sp_rank, cfg_rank) per global rank: sequence parallel fastest, then cfg."""
    if world % (sp * cfg):
        raise ValueError(f"world {world} is not a multiple of sp*cfg={sp * cfg}")
    return [(r % sp, (r // sp) % cfg) for r in range(world)]


class CfgGather:
    """Peer-store all-gather of fixed-size predictions over one cfg group."""

    def __init__(self, nbytes_per_rank: int, *, device: torch.device, group=None, rank: int = 0,
                 world: int = 1, generation: int = 0) -> None:
        import torch.distributed as dist

        if group is not None or (world > 1 and dist.is_initialized()):
            world = dist.get_world_size(group)
        self.windows = PeerWindows(nbytes_per_rank * max(world, 1) + 256, device=device,
                                   group=group, rank=rank, world=world, generation=generation)
        self.world, self.rank, self.device = self.windows.world, self.windows.rank, device
        self.slice_bytes = nbytes_per_rank
        self.offset = self.windows.carve(nbytes_per_rank * self.world)

    def __call__(self, local: torch.Tensor) -> torch.Tensor:
        local = local.contiguous()
        nbytes = local.numel() * local.element_size()
        if nbytes != self.slice_bytes:
            raise ValueError(f"gather planned for {self.slice_bytes} bytes per rank, got {nbytes}")
        stream = torch.cuda.current_stream(self.device)
        _lib.check(_lib.load().dgxm_comm_allgather(self.windows._handle, local.data_ptr(), nbytes,
                                                    self.offset, stream.cuda_stream),
                   "dgxm_comm_allgather")
        full = self.windows.local_tensor(self.offset, (self.world * local.shape[0], *local.shape[1:]),
                                         local.dtype)
        return full.clone()

    def close(self) -> None:
        self.windows.close()


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
