"""Per-conditioning CFG dispatch: conditionings that cannot share one model
call are spread over the cfg ranks, and their outputs come back over NVLink.

When ComfyUI cannot batch a step's conditionings into one call (different
text lengths, per-cond constants), the batch split of `cfg.take_slice` has
nothing to split.  The reference then gives each cfg rank a contiguous group
of condition indices, masks the others with None (stock `_calc_cond_batch`
leaves a masked output at zeros) and all-gathers the outputs back into the
sampler's order (adapters/cfg_dispatch.py:209-271).  Here the gather is the
peer-store `CfgGather` (dgxm_comm_allgather): each rank's stacked group lands
in every rank's window in rank order, which is the original cond order
because the groups are contiguous.

The path is chosen from facts every rank holds (the cond list, the cfg
world), before any collective, so no rank enters a gather another skipped.
"""
from __future__ import annotations

import contextlib
import math

import torch

# Keys a conditioning can carry that narrow or drop it for a step; the fold
# rule below does not model them, so a cond carrying one keeps the batch split
# (adapters/cfg_dispatch.py:37-41).
UNMODELLED_COND_KEYS = ("default", "area", "mask", "gligen", "timestep_start", "timestep_end")

_ABSENT = object()
_dispatching = False


def dispatch_in_progress() -> bool:
    """Whether this rank is inside its own per-cond call (the batch split
    passes such a call through: the rank owns every row of it)."""
    return _dispatching


@contextlib.contextmanager
def dispatch_scope():
    global _dispatching
    previous, _dispatching = _dispatching, True
    try:
        yield
    finally:
        _dispatching = previous


def cond_group_bounds(count: int, world: int, rank: int) -> tuple[int, int]:
    """The half-open cond-index range [start, stop) of `rank`: groups of
    ceil(count / world) in rank order, so slot j of rank r's group is global
    index r * size + j; ranks past the end own an empty range."""
    size = -(-count // world)
    start = min(rank * size, count)
    return start, min(start + size, count)


def cross_attn_pair_folds(a: int, b: int) -> bool:
    """ComfyUI's cross-attention length rule for two conditionings: equal
    lengths batch; unequal ones batch when the shorter repeats at most four
    times into their least common multiple."""
    if a == b:
        return True
    short, long_ = min(a, b), max(a, b)
    return short > 0 and math.lcm(short, long_) // short <= 4


def _entries(conds) -> list[dict]:
    """Every conditioning dict of the step, over all slots."""
    out = []
    for slot in conds or []:
        if slot:
            out.extend(item for item in slot if isinstance(item, dict))
    return out


def _constant(item: dict, key: str):
    found = (item.get("model_conds") or {}).get(key)
    return _ABSENT if found is None else getattr(found, "cond", _ABSENT)


def conds_fold(conds, x_in: torch.Tensor, key: str | None = None) -> bool:
    """Whether the step's conditionings batch into one model call, each judged
    against the first (adapters/cfg_dispatch.py:167-206): a family's declared
    constant decides first; then any key the rule does not model, any hook
    group or a control object other than the first's keeps the batch split;
    otherwise every cond object must answer `can_concat` for its processed
    value."""
    items = _entries(conds)
    if len(items) < 2:
        return True
    if key is not None:
        first = _constant(items[0], key)
        if any(not (value is first or value == first) for value in (_constant(i, key) for i in items)):
            return False
    if any(name in item for item in items for name in UNMODELLED_COND_KEYS):
        return True
    if any(item.get("hooks") is not None for item in items):
        return True
    control = items[0].get("control")
    if any(item.get("control") is not control for item in items):
        return True
    models = [item.get("model_conds") for item in items]
    readable = all(isinstance(m, dict) and all(hasattr(c, "process_cond") and hasattr(c, "can_concat")
                                               for c in m.values()) for m in models)
    if not readable:
        return True
    batch = int(x_in.shape[0])
    base = models[0]
    for other in models[1:]:
        if other.keys() != base.keys():
            return False
        for name, obj in base.items():
            mine = obj.process_cond(batch_size=batch, area=None)
            theirs = other[name].process_cond(batch_size=batch, area=None)
            if not mine.can_concat(theirs):
                return False
    return True


class CondDispatch:
    """The CALC_COND_BATCH wrapper of one cfg group.

    `gather(local)` all-gathers a (size, *x_in.shape) stack over the cfg
    ranks in rank order (a `cfg.CfgGather` for the stack's byte size, or any
    callable with that contract); `key` is the family's batch constant."""

    def __init__(self, *, world: int, rank: int, gather, key: str | None = None) -> None:
        self.world, self.rank, self.gather, self.key = world, rank, gather, key
        self.last_path: str | None = None

    def __call__(self, executor, conds, x_in, *args, **kwargs):
        present = [i for i, slot in enumerate(conds) if slot]
        if self.world <= 1 or len(present) < 2 or conds_fold(conds, x_in, self.key):
            self.last_path = "slice"
            return executor(conds, x_in, *args, **kwargs)
        self.last_path = "dispatch"
        count = len(conds)
        start, stop = cond_group_bounds(count, self.world, self.rank)
        mine = [slot if start <= i < stop else None for i, slot in enumerate(conds)]
        with dispatch_scope():
            local = executor(mine, x_in, *args, **kwargs)
        size = -(-count // self.world)
        # Every output is zeros_like(x_in) to start with, so the slots share a
        # shape; a rank with fewer than `size` conds pads with zeros.
        slots = list(local[start:stop]) + [torch.zeros_like(x_in) for _ in range(size - (stop - start))]
        gathered = self.gather(torch.stack(slots))
        return [gathered[i] for i in range(count)]
