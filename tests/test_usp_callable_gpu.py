"""The drop-in usp_attention callable at world 1 (one GPU): the reference's
surface (adapters/base.py:216-326) -- reshape modes, GQA, pad exclusion and
typed refusals -- on the B200 kernels."""
from __future__ import annotations

import pytest
import torch

from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, reference_attention, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture
def attn(lib):
    from dgx_monarch_b200.usp import make_b200_usp_attention

    return make_b200_usp_attention()


def _qkv(b, l, h, hkv, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(b, l, h, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(b, l, hkv, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(b, l, hkv, 128, device="cuda", generator=g).bfloat16()
    return q, k, v


def test_comfy_layout_round_trip(attn):
    q, k, v = _qkv(2, 500, 4, 4, 0)
    out = attn(q.reshape(2, 500, -1), k.reshape(2, 500, -1), v.reshape(2, 500, -1), heads=4)
    assert out.shape == (2, 500, 512)
    ref, _ = reference_attention(q, k, v)
    assert rel_l2(out.reshape(2, 500, 4, 128), ref) <= BF16_REL_L2


def test_skip_reshape_surfaces(attn):
    q, k, v = _qkv(1, 300, 2, 2, 1)
    out = attn(*(t.transpose(1, 2) for t in (q, k, v)), heads=2, skip_reshape=True,
               skip_output_reshape=True)
    assert out.shape == (1, 2, 300, 128)
    ref, _ = reference_attention(q, k, v)
    assert rel_l2(out.transpose(1, 2), ref) <= BF16_REL_L2


def test_native_gqa(attn):
    q, k, v = _qkv(1, 400, 8, 2, 2)
    out = attn(q.reshape(1, 400, -1), k.reshape(1, 400, -1), v.reshape(1, 400, -1), heads=8,
               enable_gqa=True)
    ref, _ = reference_attention(q, k, v)
    assert rel_l2(out.reshape(1, 400, 8, 128), ref) <= BF16_REL_L2


def test_pad_rows_are_excluded_and_zeroed(attn):
    q, k, v = _qkv(1, 140, 2, 2, 3)
    drop = [5, 139]
    out = attn(*(t.transpose(1, 2) for t in (q, k, v)), heads=2, skip_reshape=True,
               skip_output_reshape=True, drop_rows=drop).transpose(1, 2)
    keep = [i for i in range(140) if i not in drop]
    ref, _ = reference_attention(q[:, keep], k[:, keep], v[:, keep])
    assert (out[:, keep].float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert torch.equal(out[:, drop], torch.zeros_like(out[:, drop]))


def test_typed_refusals(attn):
    from dgx_monarch_b200.usp import UnsupportedModelError

    q, k, v = _qkv(1, 64, 2, 1, 4)
    flat = [t.reshape(1, 64, -1) for t in (q, k, v)]
    with pytest.raises(UnsupportedModelError, match="enable_gqa"):
        attn(*flat, heads=2)
    mask = torch.zeros(1, 1, 64, 64, device="cuda")
    mask[..., 0] = -1e9
    q2 = q.reshape(1, 64, -1)
    with pytest.raises(UnsupportedModelError, match="mask"):
        attn(q2, q2, q2, heads=2, mask=mask)
    # A no-op mask is dropped exactly, as in the reference.
    attn(q2, q2, q2, heads=2, mask=torch.zeros(1, 1, 64, 64, device="cuda"))
    with pytest.raises(UnsupportedModelError, match="cover 10 of 64"):
        attn(q2, q2, q2, heads=2, query_bias_groups=[(0, 10, None)])
    with pytest.raises(UnsupportedModelError, match="does not broadcast"):
        attn(q2, q2, q2, heads=2, query_bias_groups=[(0, 64, torch.zeros(1, 1, 3, 64, device="cuda"))])
    with pytest.raises(UnsupportedModelError, match="carries 64 rows"):
        attn(*(t.transpose(1, 2) for t in (q, q, q)), heads=2, skip_reshape=True, drop_rows=[64])


def test_invalidate_retires_the_implementation(attn):
    from dgx_monarch_b200.usp import UnsupportedModelError

    q = torch.randn(1, 32, 256, device="cuda").bfloat16()
    attn.impl.invalidate()
    with pytest.raises(UnsupportedModelError, match="retired"):
        attn(q, q, q, heads=2)


def ltx_guide_groups(tokens, guide_start, weights):
    """The LTX guide layout (tests/test_usp_query_bias.py:51-86 of the
    reference): log weights as a key row for the noisy queries and as one
    weight per tracked query row over the noisy keys; finfo.min at weight 0."""
    finfo = torch.finfo(weights.dtype)
    log_w = torch.full_like(weights, finfo.min)
    log_w[weights > 0] = torch.log(weights[weights > 0])
    tracked = weights.shape[0]
    noisy = torch.zeros((1, 1, 1, tokens), dtype=weights.dtype, device=weights.device)
    noisy[..., guide_start:guide_start + tracked] = log_w.view(1, 1, 1, -1)
    rect = torch.zeros((1, 1, tracked, tokens), dtype=weights.dtype, device=weights.device)
    rect[..., :guide_start] = log_w.view(1, 1, -1, 1)
    groups = [(0, guide_start, noisy), (guide_start, guide_start + tracked, rect)]
    if guide_start + tracked < tokens:
        groups.append((guide_start + tracked, tokens, None))
    return groups


def oracle_grouped(q, k, v, drop, groups):
    """The oracle's grouped attention with pad exclusion, float64, as a tensor."""
    from oracle import usp as oracle_usp

    host = [t.double().cpu().numpy() for t in (q, k, v)]
    g64 = [(s, e, None if b is None else b.double().cpu().numpy()) for s, e, b in groups]
    out = oracle_usp.attend_groups_without_pads(*host, drop, drop, g64)
    return torch.from_numpy(out).to(q.device)


def test_query_bias_groups_ltx_guides_and_tail_pads(attn):
    """LTX guide rectangles (per-token weights, one of them 0) on a stream
    with tail pads, against the oracle of adapters/usp_query_bias.py."""
    real, pad, heads = 700, 20, 4
    q, k, v = _qkv(1, real + pad, heads, heads, 8)
    g = torch.Generator(device="cuda").manual_seed(9)
    weights = torch.rand(150, device="cuda", generator=g) + 0.1
    weights[7] = 0.0
    weights[8] = 1.0
    groups = ltx_guide_groups(real, 520, weights)
    drop = list(range(real, real + pad))
    out = attn(*(t.transpose(1, 2) for t in (q, k, v)), heads=heads, skip_reshape=True,
               skip_output_reshape=True, drop_rows=drop, query_bias_groups=groups).transpose(1, 2)
    want = oracle_grouped(q, k, v, drop, groups)
    assert (out[:, :real].double() - want[:, :real]).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(out[:, :real], want[:, :real].float()) <= BF16_REL_L2
    assert torch.equal(out[:, real:], torch.zeros_like(out[:, real:]))


def test_query_bias_lens_key_row_and_per_head_bias(attn):
    """One group carrying a key bias narrower than the key axis (the Lens
    joint-attention form), and a per-head key bias in a later group."""
    rows, heads = 400, 2
    q, k, v = _qkv(1, rows, heads, heads, 10)
    g = torch.Generator(device="cuda").manual_seed(12)
    lens = [(0, rows, torch.randn(1, 1, 1, 330, device="cuda", generator=g))]
    out = attn(*(t.reshape(1, rows, -1) for t in (q, k, v)), heads=heads,
               query_bias_groups=lens).reshape(1, rows, heads, 128)
    assert rel_l2(out, oracle_grouped(q, k, v, None, lens).float()) <= BF16_REL_L2
    per_head = [(0, 150, None), (150, rows, torch.randn(1, heads, 1, rows, device="cuda", generator=g))]
    out = attn(*(t.reshape(1, rows, -1) for t in (q, k, v)), heads=heads,
               query_bias_groups=per_head).reshape(1, rows, heads, 128)
    assert rel_l2(out, oracle_grouped(q, k, v, None, per_head).float()) <= BF16_REL_L2


def test_query_bias_refusals(attn):
    from dgx_monarch_b200.usp import UnsupportedModelError

    q, k, v = _qkv(1, 64, 2, 2, 14)
    qs = [t.transpose(1, 2) for t in (q, k, v)]
    groups = [(0, 60, torch.zeros(1, 1, 1, 60, device="cuda"))]
    with pytest.raises(UnsupportedModelError, match="away from the tail"):
        attn(*qs, heads=2, skip_reshape=True, drop_rows=[3, 63, 62, 61], query_bias_groups=groups)
    many = [(i, i + 1, torch.zeros(1, 1, 1, 64, device="cuda")) for i in range(64)]
    with pytest.raises(UnsupportedModelError, match="at most"):
        attn(*qs, heads=2, skip_reshape=True, query_bias_groups=many)


def test_fp8_callable_on_one_rank(lib):
    """The FP8 drop-in at Ulysses degree 1 quantises the caller's heads in
    place of a scatter (per-head e4m3 scales) and attends them."""
    from dgx_monarch_b200.usp import make_b200_usp_attention

    attn = make_b200_usp_attention(fp8=True)
    q, k, v = _qkv(2, 640, 4, 4, 21)
    for _ in range(2):  # the second call reuses the e4m3 buffers
        out = attn(*(t.reshape(2, 640, -1) for t in (q, k, v)), heads=4).reshape(2, 640, 4, 128)
    from tests.test_attn_gpu import FP8_REL_L2, fp8_references

    ref, _ = reference_attention(q, k, v)
    ref_deq, floor = fp8_references(q, k, v)  # per-head scales over both batch rows, as the drop-in takes
    assert rel_l2(out, ref_deq) <= FP8_REL_L2
    assert rel_l2(out, ref) <= floor + FP8_REL_L2  # e4m3 inputs against bf16 activations
    attn.impl.invalidate()


def test_fp8_callable_excludes_pad_rows(lib):
    """FP8 with divisibility pads at Ulysses degree 1: as the reference hands
    its inner kernel the real rows only (adapters/usp_pad_exclusion.py:112-137),
    pad rows neither attend nor set a head's e4m3 scale, and come back as
    zeros."""
    from dgx_monarch_b200.usp import make_b200_usp_attention
    from tests.test_attn_gpu import FP8_REL_L2, fp8_references

    attn = make_b200_usp_attention(fp8=True)
    q, k, v = _qkv(1, 640, 4, 4, 22)
    drop = list(range(632, 640))
    q, k, v = (t.clone() for t in (q, k, v))
    for t in (q, k, v):
        t[:, drop] = 40.0  # pad content far outside the real rows' range
    out = attn(*(t.reshape(1, 640, -1) for t in (q, k, v)), heads=4, drop_rows=drop).reshape(1, 640, 4, 128)
    real = slice(0, 632)
    ref_deq, _ = fp8_references(q[:, real], k[:, real], v[:, real])
    assert rel_l2(out[:, real], ref_deq) <= FP8_REL_L2
    assert torch.count_nonzero(out[:, drop]).item() == 0
    attn.impl.invalidate()


@pytest.mark.parametrize("head_dim", [64, 96])
def test_small_head_dims_run_zero_padded(attn, head_dim):
    """Heads below 128 (LTX-Video's 64) run zero-padded with the scale of their
    own head dimension: plain, and with LTX guide biases on tail pads."""
    real, pad, heads = 700, 20, 4
    g = torch.Generator(device="cuda").manual_seed(head_dim)
    q, k, v = (torch.randn(1, real + pad, heads, head_dim, device="cuda", generator=g).bfloat16()
               for _ in range(3))
    out = attn(*(t.reshape(1, real + pad, -1) for t in (q, k, v)), heads=heads)
    assert out.shape == (1, real + pad, heads * head_dim)
    ref, _ = reference_attention(q, k, v)
    got = out.reshape(1, real + pad, heads, head_dim)
    assert (got.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(got, ref) <= BF16_REL_L2

    weights = torch.rand(150, device="cuda", generator=g) + 0.1
    groups = ltx_guide_groups(real, 520, weights)
    drop = list(range(real, real + pad))
    out = attn(*(t.transpose(1, 2) for t in (q, k, v)), heads=heads, skip_reshape=True,
               skip_output_reshape=True, drop_rows=drop, query_bias_groups=groups).transpose(1, 2)
    want = oracle_grouped(q, k, v, drop, groups)
    assert out.shape == (1, real + pad, heads, head_dim)
    assert (out[:, :real].double() - want[:, :real]).abs().max().item() <= BF16_MAX_ABS
    assert torch.equal(out[:, real:], torch.zeros_like(out[:, real:]))
