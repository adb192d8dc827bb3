"""Pin the CPU oracle to golden vectors produced by the reference itself.

tests/golden/make_golden.py ran the reference's own modules (with the
third-party leaves stubbed as its tests stub them) and recorded inputs and
outputs.  Integer and permutation results must match exactly; float64
attention results to 1e-12.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import usp

GOLDEN = Path(__file__).resolve().parent / "golden"
SPEC = json.loads((GOLDEN / "golden.json").read_text())
ARR = np.load(GOLDEN / "golden_arrays.npz")


@pytest.mark.parametrize("case", SPEC["padded_row_indices"], ids=lambda c: f"w{c['world']}-{c['segments'][:2]}")
def test_padded_row_indices_match_reference(case):
    segs = [tuple(s) for s in case["segments"]]
    assert usp.padded_row_indices(segs, case["world"]) == case["rows"]


def test_hand_computed_krea2_geometries():
    """The literal layouts of the reference's tests/test_usp_pad_exact.py:28-75."""
    assert usp.padded_row_indices([(512, 256), (9216, 4608)], 2) == []
    assert usp.padded_row_indices([(512, 256), (8281, 4141)], 2) == [8793]
    assert usp.padded_row_indices([(511, 256), (8281, 4141)], 2) == [4652, 8793]
    assert usp.padded_row_indices([(512, 256), (8275, 4139)], 2) == [8787, 8788, 8789]
    last = 3 * (128 + 2071)
    assert usp.padded_row_indices([(510, 128), (8281, 2071)], 4) == [
        last + 126, last + 127, last + 128 + 2071 - 3, last + 128 + 2071 - 2, last + 128 + 2071 - 1]


@pytest.mark.parametrize("case", SPEC["joint_order"], ids=lambda c: f"{c['text']}-{c['image']}-{c['world']}")
def test_joint_order_matches_reference(case):
    order = usp.RankMajorJointOrder(case["text"], case["image"])
    rows = case["world"] * (case["text"] + case["image"])
    assert order.permutation(rows).tolist() == case["permutation"]
    z = np.zeros((1, rows, 1, 1))
    _q, _k, _v, qd, kd, perm = order.canonicalize(z, z, z, case["drop"], case["kv_drop"])
    assert qd == case["canon_drop"] and kd == case["canon_kv_drop"]
    x = np.arange(rows, dtype=np.float64).reshape(1, rows, 1, 1)
    assert np.array_equal(order.restore(x[:, perm], perm), x)


def test_joint_order_literal_round_trip():
    """tests/test_usp_sequence_order.py:10-20 of the reference, verbatim values."""
    order = usp.RankMajorJointOrder(3, 5)
    q = np.arange(16, dtype=np.float32).reshape(1, 16, 1, 1)
    cq, _, _, drop, kv_drop, perm = order.canonicalize(q, q, q, [7, 15], [2, 11])
    assert cq[0, :, 0, 0].tolist() == [0, 1, 2, 8, 9, 10, 3, 4, 5, 6, 7, 11, 12, 13, 14, 15]
    assert drop == [10, 15] and kv_drop == [2, 11]


@pytest.mark.parametrize("case", SPEC["keep_index"], ids=lambda c: f"{c['rows']}-{c['drop']}")
def test_keep_index_matches_reference(case):
    got = usp.kept_rows(case["rows"], case["drop"])
    assert (None if got is None else got.tolist()) == case["kept"]


def test_keep_index_refuses_out_of_range_rows():
    with pytest.raises(usp.OracleRefusal, match="carries 118 rows"):
        usp.kept_rows(118, [7905])
    with pytest.raises(usp.OracleRefusal):
        usp.kept_rows(4, [-1])


def _attend64(q, k, v):
    return usp.attention_lse(q, k, v)[0]


@pytest.mark.parametrize("case", SPEC["full_axis"], ids=lambda c: str(c["index"]))
def test_full_axis_composition_matches_reference(case):
    """Canonicalize -> drop pads -> attend -> restore, as run_full_axis does
    (adapters/usp_full_axis.py:9-40), with the gathered axis handed in."""
    n = case["index"]
    gathered = ARR[f"full_axis_{n}_in"]
    order = usp.RankMajorJointOrder(case["text"], case["image"])
    q, k, v, qd, kd, perm = order.canonicalize(gathered, gathered, gathered, case["drop"], case["kv_drop"])
    out = usp.attend_without_pads(q, k, v, qd or None, kd or None, _attend64)
    out = order.restore(out, perm)
    np.testing.assert_allclose(out, ARR[f"full_axis_{n}_sent"], atol=1e-12, rtol=0)
    np.testing.assert_allclose(out, ARR[f"full_axis_{n}_out"], atol=1e-12, rtol=0)


@pytest.mark.parametrize("case", SPEC["usp_callable"], ids=lambda c: str(c["index"]))
def test_usp_callable_world1_matches_reference(case):
    """Reshape, GQA repeat and pad exclusion of adapters/base.py:216-326."""
    n = case["index"]
    q, k, v = (ARR[f"callable_{n}_{x}"] for x in "qkv")
    drop = case["drop"]
    out = usp.attend_without_pads(q, k, v, drop, drop, _attend64)
    np.testing.assert_allclose(out, ARR[f"callable_{n}_out"], atol=1e-12, rtol=0)


@pytest.mark.parametrize("case", SPEC["cfg_slice"], ids=lambda c: f"{c['world']}-{c['rank']}")
def test_cfg_slice_matches_reference(case):
    w, r = case["world"], case["rank"]
    tree = {"x": ARR["cfg_in_x"], "nested": [ARR["cfg_in_x"][:, 0], ARR["cfg_in_bcast"]]}
    got = usp.cfg_take_slice(tree, 4, w, r)
    assert np.array_equal(got["x"], ARR[f"cfg_{w}_{r}_x"])
    assert np.array_equal(got["nested"][0], ARR[f"cfg_{w}_{r}_n0"])
    assert np.array_equal(got["nested"][1], ARR[f"cfg_{w}_{r}_n1"])


@pytest.mark.parametrize("case", SPEC["shard_seq"], ids=lambda c: f"{c['world']}-{c['rank']}")
def test_shard_seq_matches_reference(case):
    local, orig = usp.shard_seq(ARR["shard_in"], case["world"], case["rank"])
    assert orig == case["orig"]
    assert np.array_equal(local, ARR[f"shard_{case['world']}_{case['rank']}"])


def test_shard_then_gather_round_trips():
    t = ARR["shard_in"]
    for world in (2, 3, 4):
        chunks = [usp.shard_seq(t, world, r)[0] for r in range(world)]
        assert np.array_equal(usp.sp_gather(chunks, t.shape[1]), t)


@pytest.mark.parametrize("case", SPEC["probe"], ids=lambda c: c["dtype"])
def test_known_answer_probe_matches_reference_formula(case):
    """The dyadic probe of adapters/cudnn_ring_attention.py:106-135."""
    n = case["index"]
    q, k, v = (ARR[f"probe_{n}_{x}"] for x in "qkv")
    out, lse = usp.attention_lse(q, k, v, case["scale"])
    np.testing.assert_allclose(lse, ARR[f"probe_{n}_lse"], atol=2e-5, rtol=2e-5)
    eps = 2.0 ** -7 if "bfloat16" in case["dtype"] else 2.0 ** -10
    np.testing.assert_allclose(out, ARR[f"probe_{n}_out"], atol=eps, rtol=2 * eps)


def test_ring_merge_equals_full_attention():
    rng = np.random.default_rng(0)
    world = 4
    q = [rng.standard_normal((1, 6, 2, 8)) for _ in range(world)]
    k = [rng.standard_normal((1, 6, 2, 8)) for _ in range(world)]
    v = [rng.standard_normal((1, 6, 2, 8)) for _ in range(world)]
    ring = usp.ring_attention(q, k, v)
    K, V = np.concatenate(k, 1), np.concatenate(v, 1)
    for r in range(world):
        ref_out, ref_lse = usp.attention_lse(q[r], K, V)
        np.testing.assert_allclose(ring[r][0], ref_out, atol=1e-12)
        np.testing.assert_allclose(ring[r][1], ref_lse, atol=1e-12)


def test_ulysses_equals_unsharded_attention():
    rng = np.random.default_rng(1)
    world, rows, heads = 4, 24, 8
    q, k, v = (rng.standard_normal((1, rows, heads, 8)) for _ in range(3))
    chunk = rows // world
    split = lambda t: [t[:, r * chunk:(r + 1) * chunk] for r in range(world)]
    outs = usp.ulysses_attention(split(q), split(k), split(v))
    np.testing.assert_allclose(np.concatenate(outs, 1), usp.attention_lse(q, k, v)[0], atol=1e-12)


def test_all_to_all_round_trip_is_identity_and_rank_major():
    rng = np.random.default_rng(2)
    world = 4
    local = [rng.standard_normal((2, 5, 8, 3)) for _ in range(world)]
    scattered = usp.seq_all_to_all_4d(local, 2, 1)
    for r in range(world):
        assert scattered[r].shape == (2, 20, 2, 3)
        for s in range(world):  # rank-major: source s's rows land at [s*5, (s+1)*5)
            assert np.array_equal(scattered[r][:, s * 5:(s + 1) * 5], local[s][:, :, 2 * r:2 * r + 2])
    back = usp.seq_all_to_all_4d(scattered, 1, 2)
    for r in range(world):
        assert np.array_equal(back[r], local[r])


def test_hybrid_groups_are_ulysses_low():
    uly, ring = usp.hybrid_groups(8, 2, 4)
    assert uly == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert ring == [[0, 2, 4, 6], [1, 3, 5, 7]]


def _bias_groups(case):
    return [(start, end, None if name is None else ARR[name]) for start, end, name in case["groups"]]


@pytest.mark.parametrize("case", SPEC["query_bias"], ids=lambda c: c["name"])
def test_query_bias_groups_match_reference(case):
    """Query-group biases through the reference's callable
    (adapters/usp_query_bias.py:109-130, with pads adapters/usp_pad_exclusion.py:112-137)."""
    name = case["name"]
    q, k, v = (ARR[f"bias_{name}_{x}"] for x in "qkv")
    drop = case["drop"]
    out = usp.attend_groups_without_pads(q, k, v, drop, drop, _bias_groups(case))
    np.testing.assert_allclose(out, ARR[f"bias_{name}_out"], atol=1e-12, rtol=0)


@pytest.mark.parametrize("groups,reason", [
    (((0, 4, None), (6, 10, None)), "gap"),
    (((0, 6, None), (4, 10, None)), "overlap"),
    (((0, 6, None),), "short"),
    (((0, 12, None),), "past the end"),
    (((0, 10, np.zeros((1, 1, 3, 10))),), "rows"),
    (((0, 10, np.zeros((1, 1, 1, 40))),), "keys"),
])
def test_malformed_bias_groups_refuse(groups, reason):
    with pytest.raises(usp.OracleRefusal):
        usp.validate_query_bias_groups(groups, 10, 10)


def test_bias_pads_must_be_a_tail():
    usp.assert_pads_are_a_tail([12, 13], 14)
    with pytest.raises(usp.OracleRefusal, match="away from the tail"):
        usp.assert_pads_are_a_tail([3, 13], 14)


@pytest.mark.parametrize("case", SPEC["full_context"], ids=lambda c: str(c["index"]))
def test_full_context_gather_matches_reference(case):
    """The reference's Ring2 K/V gather on a gloo world-2 group
    (adapters/wan_ring_full_context.py:203-295): rank-major slots, the same
    gathered axis on both ranks."""
    n = case["index"]
    for name in "kv":
        blocks = [ARR[f"fullctx_{n}_{name}{r}"] for r in range(2)]
        want = usp.full_context_gather(blocks)
        for r in range(2):
            np.testing.assert_array_equal(ARR[f"fullctx_{n}_full{name}{r}"], want)


def test_full_context_equals_ring_merge():
    """Local-Q x full-KV in one softmax equals the ring's per-block merge."""
    rng = np.random.default_rng(11)
    q, k, v = ([rng.standard_normal((1, 6, 2, 8)) for _ in range(3)] for _ in range(3))
    full = usp.full_context_ring_attention(q, k, v)
    ring = usp.ring_attention(q, k, v)
    for (o1, l1), (o2, l2) in zip(full, ring):
        np.testing.assert_allclose(o1, o2, atol=1e-12, rtol=0)
        np.testing.assert_allclose(l1, l2, atol=1e-12, rtol=0)


@pytest.mark.parametrize("case", SPEC["shared_scale"], ids=lambda c: f"{c['dtype']}-w{c['world']}")
def test_shared_activation_scale_matches_reference(case):
    """The reference's shared NVFP4 scale with a replay reducer
    (adapters/quant_activation_scale.py:222-246): every shard gets the
    one-GPU scale of the whole tensor."""
    n = case["index"]
    x = ARR[f"scale_{n}_x"]
    shards = np.array_split(x, case["world"], axis=0)
    want = usp.shared_activation_scale(shards, case["divisor"], case["dtype"])
    for got in ARR[f"scale_{n}_out"]:
        assert np.float32(got) == np.float32(want)


def test_round_to_bf16_is_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.01171875, 3.0e38, -2.5e-3, np.inf, np.nan], dtype=np.float32)
    got = usp.round_to_bf16(vals)
    assert got[1] == 1.0                      # a tie rounds to the even mantissa
    assert got[2] == np.float32(1.015625)     # a tie rounds up to the even neighbour
    assert np.isinf(got[5]) and np.isnan(got[6])
