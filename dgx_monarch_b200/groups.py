"""Process-group layout of a Ulysses x ring sequence-parallel world.

The reference builds its groups through xfuser's initialize_model_parallel
(actor/worker_env.py:320-327), which hands yunchang the "ulysses-low"
layout: a Ulysses group is a run of consecutive ranks (so its all-to-all
stays between neighbouring GPUs) and a ring group takes one rank from each
Ulysses group of the same sequence-parallel block.  No reference test pins
this layout (its tests stub xfuser); the layout here is that assumption,
written once for the package and checked against the oracle's restatement.
"""
from __future__ import annotations


def hybrid_layout(world: int, ulysses: int, ring: int) -> tuple[list[list[int]], list[list[int]]]:
    """(Ulysses groups, ring groups) as lists of global ranks.

    Rank g of sequence-parallel block b = g // (ulysses * ring) sits at
    Ulysses position g % ulysses and ring position (g // ulysses) % ring."""
    if ulysses < 1 or ring < 1:
        raise ValueError(f"ulysses {ulysses} and ring {ring} must be positive")
    sp = ulysses * ring
    if world % sp:
        raise ValueError(f"world {world} is not a multiple of ulysses*ring={sp}")
    uly_groups = [list(range(start, start + ulysses)) for start in range(0, world, ulysses)]
    ring_groups = [[block + u + ulysses * i for i in range(ring)]
                   for block in range(0, world, sp) for u in range(ulysses)]
    return uly_groups, ring_groups


def new_hybrid_groups(world: int, ulysses: int, ring: int, **kwargs):
    """Create every Ulysses and ring group of the layout (collective: every
    rank creates every group, in the same order) and return this rank's
    (Ulysses group, ring group).  kwargs go to torch.distributed.new_group."""
    import torch.distributed as dist

    uly_groups, ring_groups = hybrid_layout(world, ulysses, ring)
    rank = dist.get_rank()
    mine = {}
    for kind, groups in (("ulysses", uly_groups), ("ring", ring_groups)):
        for ranks in groups:
            group = dist.new_group(ranks, **kwargs)
            if rank in ranks:
                mine[kind] = group
    return mine["ulysses"], mine["ring"]
