"""Host logic of the usp_attention drop-in, on the CPU: head dimensions below
the kernels' 128 are zero-padded with the softmax scale of the real head
dimension, and the output is trimmed back; unsupported head dimensions are
refused before any device work.  The implementation's `attend` is replaced by
the float64 oracle, so only the callable's own reshapes, padding, scale and
trimming are under test here (the kernels are tested on the GPU)."""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import usp as oracle


def _callable_with_oracle_attend(seen, head_dim):
    """A CPU callable whose attend records its arguments and runs the oracle."""
    from dgx_monarch_b200.usp import make_b200_usp_attention

    attn = make_b200_usp_attention(device=torch.device("cpu"))

    def attend(q, k, v, drop_rows, kv_rows, order, groups, softmax_scale=None):
        seen.append({"shape": tuple(q.shape), "kv_shape": tuple(k.shape), "scale": softmax_scale,
                     "dtype": q.dtype,
                     "pad_max": max(float(t[..., head_dim:].abs().max()) if t.shape[-1] > head_dim else 0.0
                                    for t in (q, k, v))})
        out, _ = oracle.attention_lse(q.double().numpy(), k.double().numpy(), v.double().numpy(),
                                      scale=softmax_scale)
        return torch.from_numpy(out).to(torch.bfloat16)

    attn.impl.attend = attend
    return attn


@pytest.mark.parametrize("head_dim,heads,kv_heads,runs_at", [
    (40, 2, 2, 64), (64, 4, 4, 64), (72, 3, 3, 128), (96, 4, 2, 128), (128, 2, 2, 128)])
def test_small_heads_are_padded_with_their_own_scale(head_dim, heads, kv_heads, runs_at):
    """Head dimensions up to 64 run at the kernel's 64, larger ones at 128;
    the padding is zeros and the scale stays that of the caller's head_dim."""
    seen = []
    attn = _callable_with_oracle_attend(seen, head_dim)
    g = torch.Generator().manual_seed(head_dim)
    q = torch.randn(1, 40, heads * head_dim, generator=g)
    k = torch.randn(1, 40, kv_heads * head_dim, generator=g)
    v = torch.randn(1, 40, kv_heads * head_dim, generator=g)
    out = attn(q, k, v, heads=heads, enable_gqa=kv_heads != heads)
    (call,) = seen
    assert call["shape"] == (1, 40, heads, runs_at)
    assert call["kv_shape"][-1] == runs_at
    assert call["dtype"] == torch.bfloat16
    assert call["pad_max"] == 0.0
    assert call["scale"] == pytest.approx(1.0 / math.sqrt(head_dim))
    assert out.shape == q.shape and out.dtype == q.dtype
    # One-process attention over the bf16-rounded, unpadded inputs.
    qb, kb, vb = (t.bfloat16().double().reshape(1, 40, -1, head_dim).numpy() for t in (q, k, v))
    want, _ = oracle.attention_lse(qb, kb, vb)
    got = out.reshape(1, 40, heads, head_dim).double().numpy()
    assert np.abs(got - want).max() <= 2e-2


@pytest.mark.parametrize("head_dim", [130, 256, 60, 4])
def test_unsupported_head_dims_are_refused(head_dim):
    from dgx_monarch_b200.usp import UnsupportedModelError

    seen = []
    attn = _callable_with_oracle_attend(seen, head_dim)
    x = torch.zeros(1, 8, 2 * head_dim)
    with pytest.raises(UnsupportedModelError, match=f"head_dim {head_dim}"):
        attn(x, x, x, heads=2)
    assert not seen


def _unpack(bits: torch.Tensor, rows: int) -> np.ndarray:
    words = bits.numpy().astype(np.uint32)
    return np.array([(int(words[i // 32]) >> (i % 32)) & 1 for i in range(rows)], dtype=bool)


@pytest.mark.parametrize("rows,drop", [(140, [5, 139]), (64, [0, 31, 32, 63]), (1216, list(range(1200, 1216))),
                                       (33, [32]), (700, [0, 5, 127, 128, 255, 256, 311, 699])])
def test_keep_bits_mark_exactly_the_oracle_kept_rows(rows, drop):
    """Bit i of word i // 32 is set exactly for the rows the oracle keeps
    (adapters/usp_pad_exclusion.py:79-126); bits past the axis stay clear."""
    from dgx_monarch_b200.ops import keep_bits

    bits = keep_bits(rows, drop, torch.device("cpu"))
    assert bits.dtype == torch.int32 and bits.numel() == (rows + 31) // 32
    kept = np.zeros(rows, dtype=bool)
    kept[oracle.kept_rows(rows, drop)] = True
    np.testing.assert_array_equal(_unpack(bits, rows), kept)
    tail = int(bits[-1].item()) & 0xFFFFFFFF
    assert tail >> (rows % 32 or 32) == 0


def test_keep_bits_are_cached_per_layout_and_device():
    """Built once per (rows, drop set, device) from host integers -- nothing is
    read back from a device -- and a cached entry equals a fresh build, as
    tests/test_usp_pad_index_cache.py pins for the reference's keep index."""
    from dgx_monarch_b200 import ops

    ops._KEEP_BITS.clear()
    first = ops.keep_bits(300, [7, 299], torch.device("cpu"))
    assert ops.keep_bits(300, [299, 7, 7], torch.device("cpu")) is first
    other = ops.keep_bits(301, [7, 299], torch.device("cpu"))
    assert other is not first
    ops._KEEP_BITS.clear()
    assert torch.equal(ops.keep_bits(300, [7, 299], torch.device("cpu")), first)
    assert ops.keep_bits(300, [], torch.device("cpu")) is None
    with pytest.raises(ValueError, match="carries 300 rows"):
        ops.keep_bits(300, [300], torch.device("cpu"))
    with pytest.raises(ValueError):
        ops.keep_bits(300, [-1], torch.device("cpu"))


_GROUP_CASES = [
    ((0, 4, None), (4, 10, None)),
    ((0, 4, None), (6, 10, None)),
    ((0, 6, None), (4, 10, None)),
    ((0, 6, None),),
    ((0, 12, None),),
    ((0, 10, np.zeros((1, 1, 3, 10))),),
    ((0, 10, np.zeros((1, 1, 1, 40))),),
    ((0, 10, np.zeros((1, 1, 1, 10))),),
    ((0, 3, np.zeros((1, 2, 3, 8))), (3, 10, None)),
]


@pytest.mark.parametrize("groups", _GROUP_CASES)
def test_bias_group_validation_agrees_with_the_oracle(groups):
    """The drop-in accepts exactly the partitions the oracle's restatement of
    adapters/usp_query_bias.py:64-92 accepts (10 queries, 20 keys)."""
    from dgx_monarch_b200.usp import UnsupportedModelError, validate_bias_groups

    as_torch = [(s, e, None if b is None else torch.from_numpy(b).float()) for s, e, b in groups]
    try:
        oracle.validate_query_bias_groups(list(groups), 10, 20)
        oracle_ok = True
    except oracle.OracleRefusal:
        oracle_ok = False
    try:
        validate_bias_groups(as_torch, 10, 20, batch=1, heads=2)
        ours_ok = True
    except UnsupportedModelError:
        ours_ok = False
    assert ours_ok == oracle_ok


def test_bias_group_validation_adds_the_kernel_limits():
    from dgx_monarch_b200.usp import UnsupportedModelError, validate_bias_groups

    with pytest.raises(UnsupportedModelError, match="broadcast over batch"):
        validate_bias_groups([(0, 4, torch.zeros(3, 1, 1, 4))], 4, 4, batch=2, heads=1)
    many = [(i, i + 1, torch.zeros(1, 1, 1, 4)) for i in range(9)]
    with pytest.raises(UnsupportedModelError, match="at most 8"):
        validate_bias_groups(many, 9, 4, batch=1, heads=1)


@pytest.mark.parametrize("drop", [[], [18, 19], [3, 10], [0, 5, 19]])
def test_rank_bias_slices_heads_and_spreads_past_interior_key_pads(drop):
    """Each rank gets its own heads of a per-head bias; a bias that names keys
    by their position among the kept keys lands on those keys of the padded
    axis (zero at the pads, which the keep bits exclude anyway)."""
    from dgx_monarch_b200.usp import _rank_bias

    keys, heads, world = 20, 4, 2
    hl = heads // world
    g = torch.Generator().manual_seed(len(drop))
    n_decl = keys - len(drop) - 2                      # declared keys, fewer than the kept ones
    bias = torch.randn(1, heads, 3, n_decl, generator=g)
    shared = torch.randn(1, 1, 1, n_decl, generator=g)
    kept = [r for r in range(keys) if r not in set(drop)]
    for rank in range(world):
        out = _rank_bias([(0, 3, bias), (3, 5, None), (5, 6, shared)], rank, hl, keys, drop)
        assert out[1] == (3, 5, None)
        for (start, end, got), src in ((out[0], bias[:, rank * hl:(rank + 1) * hl]), (out[2], shared)):
            assert got.dtype == torch.float32 and got.is_contiguous()
            if drop and drop != list(range(keys - len(drop), keys)):
                assert torch.equal(got[..., kept[:n_decl]], src)
                dropped_inside = [r for r in drop if r < got.shape[-1]]
                assert torch.count_nonzero(got[..., dropped_inside]) == 0
            else:
                assert torch.equal(got, src)


@pytest.mark.parametrize("text,image,world", [(3, 5, 2), (64, 1152, 8), (1, 1, 4), (2, 7, 3)])
def test_joint_inverse_is_the_oracle_inverse_permutation(text, image, world):
    """rank-major gathered row -> canonical row, the inverse of the oracle's
    RankMajorJointOrder permutation (adapters/usp_sequence_order.py:69-78)."""
    from dgx_monarch_b200.usp import _joint_inverse

    order = oracle.RankMajorJointOrder(text, image)
    perm = order.permutation((text + image) * world)
    assert _joint_inverse(text, image, world) == list(order.inverse(perm))


_GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "golden.json").read_text())


@pytest.mark.parametrize("entry", _GOLDEN["usp_refusals"], ids=lambda e: e["verdict"][:24])
def test_typed_refusals_match_the_reference(entry):
    """Malformed calls are refused with the reference's messages
    (adapters/base.py:216-292, recorded by make_golden.py section (m)); the
    well-formed ones reach the kernel."""
    from dgx_monarch_b200.usp import UnsupportedModelError

    case = entry["case"]
    q, k, v = (torch.zeros(case[n]) for n in "qkv")
    kwargs = dict(case["kw"])
    if case.get("mask") == "effective":
        kwargs["mask"] = torch.zeros(1, 1, 8, 8)
        kwargs["mask"][..., 0] = -1e9
    elif case.get("mask") == "noop":
        kwargs["mask"] = torch.zeros(1, 1, 8, 8)
    seen = []
    attn = _callable_with_oracle_attend(seen, q.shape[-1] // kwargs["heads"] if q.ndim == 3 else q.shape[-1])
    try:
        attn(q, k, v, **kwargs)
        said = "ok"
    except UnsupportedModelError as exc:
        said = str(exc)
    assert said == entry["verdict"]
    assert bool(seen) == (said == "ok")
