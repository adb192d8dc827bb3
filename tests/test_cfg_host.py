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


@pytest.mark.parametrize("axes", [[16, 56, 56], [0, 64, 64], [128], [32, 48, 48]])
def test_rope_table_is_the_oracle_angles_rounded_once(axes):
    """The fused prologue's (rows, 64, 2) cos/sin table is cos/sin of the
    oracle's float64 angles rounded once to fp32 (Wan 3-axis, Flux 2-axis and
    1-axis layouts)."""
    from dgx_monarch_b200.prologue import rope_table

    g = np.random.default_rng(len(axes))
    pos = g.integers(0, 90, size=(57, len(axes)))
    got = rope_table(torch.from_numpy(pos), axes).numpy()
    ang = oracle.rope_table(pos, axes)
    assert got.shape == (57, 64, 2) and got.dtype == np.float32
    # Within one fp32 ulp of 1.0: libm and torch may round the float64 cos/sin
    # differently in the last bit before the single rounding to fp32.
    np.testing.assert_allclose(got[..., 0], np.cos(ang), rtol=0, atol=2.0 ** -23)
    np.testing.assert_allclose(got[..., 1], np.sin(ang), rtol=0, atol=2.0 ** -23)


def test_rope_table_refuses_axes_that_do_not_fill_the_head():
    from dgx_monarch_b200.prologue import rope_table

    with pytest.raises(ValueError, match="sum to the head dimension"):
        rope_table(torch.zeros(4, 2), [64, 32])
