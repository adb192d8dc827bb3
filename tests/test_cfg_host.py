"""Host logic of the CFG split and sequence sharding, on the CPU, against the
golden vectors the reference itself produced (tests/golden/make_golden.py):
the per-rank batch slice of adapters/cfg_parallel.py:71-87 and the shard of
adapters/base.py:48-123, plus the rank layout of the cfg x sequence-parallel
groups against the oracle."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import usp as oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
SPEC = json.loads((GOLDEN / "golden.json").read_text())
ARR = np.load(GOLDEN / "golden_arrays.npz")


@pytest.mark.parametrize("case", SPEC["cfg_slice"], ids=lambda c: f"{c['world']}-{c['rank']}")
def test_cfg_take_slice_matches_the_reference(case):
    from dgx_monarch_b200.cfg import leading_batch, take_slice

    w, r = case["world"], case["rank"]
    x = torch.from_numpy(ARR["cfg_in_x"])
    tree = {"x": x, "nested": (x[:, 0], torch.from_numpy(ARR["cfg_in_bcast"])), "note": "kept"}
    assert leading_batch(tree) == 4
    got = take_slice(tree, 4, w, r)
    assert np.array_equal(got["x"].numpy(), ARR[f"cfg_{w}_{r}_x"])
    assert isinstance(got["nested"], tuple)
    assert np.array_equal(got["nested"][0].numpy(), ARR[f"cfg_{w}_{r}_n0"])
    assert np.array_equal(got["nested"][1].numpy(), ARR[f"cfg_{w}_{r}_n1"])
    assert got["note"] == "kept"


@pytest.mark.parametrize("case", SPEC["shard_seq"], ids=lambda c: f"{c['world']}-{c['rank']}")
def test_shard_seq_matches_the_reference(case):
    from dgx_monarch_b200.shard import shard_seq

    local, orig = shard_seq(torch.from_numpy(ARR["shard_in"]), case["world"], case["rank"])
    assert orig == case["orig"]
    assert np.array_equal(local.numpy(), ARR[f"shard_{case['world']}_{case['rank']}"])


@pytest.mark.parametrize("world,sp,cfg", [(8, 4, 2), (8, 2, 2), (4, 1, 2), (2, 2, 1), (6, 3, 2)])
def test_cfg_rank_layout_matches_the_oracle(world, sp, cfg):
    from dgx_monarch_b200.cfg import cfg_rank_layout

    want = [(e["sp_rank"], e["cfg_rank"]) for e in oracle.cfg_rank_layout(world, sp, cfg)]
    assert cfg_rank_layout(world, sp, cfg) == want


def test_cfg_rank_layout_refuses_a_world_it_does_not_tile():
    from dgx_monarch_b200.cfg import cfg_rank_layout

    with pytest.raises(ValueError):
        cfg_rank_layout(6, 4, 2)
    with pytest.raises(oracle.OracleRefusal):
        oracle.cfg_rank_layout(6, 4, 2)


def test_leading_batch_finds_the_first_tensor():
    from dgx_monarch_b200.cfg import leading_batch

    assert leading_batch([None, {"a": 3, "b": torch.zeros(5, 2)}]) == 5
    assert leading_batch({"s": torch.tensor(1.0)}) is None
    assert leading_batch(("no", "tensors")) is None
