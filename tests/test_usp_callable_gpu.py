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
    with pytest.raises(UnsupportedModelError, match="query-group"):
        attn(q2, q2, q2, heads=2, query_bias_groups=[(0, 2)])
    with pytest.raises(UnsupportedModelError, match="carries 64 rows"):
        attn(*(t.transpose(1, 2) for t in (q, q, q)), heads=2, skip_reshape=True, drop_rows=[64])


def test_invalidate_retires_the_implementation(attn):
    from dgx_monarch_b200.usp import UnsupportedModelError

    q = torch.randn(1, 32, 256, device="cuda").bfloat16()
    attn.impl.invalidate()
    with pytest.raises(UnsupportedModelError, match="retired"):
        attn(q, q, q, heads=2)
