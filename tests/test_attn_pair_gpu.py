"""Attention on CTA pairs, the library default for 16-bit inputs at head dim
128: clusters of two CTAs on one TPC, each CTA loading half of every K/V block
(64 keys of K, 64 head dimensions of V) and one thread issuing the M256
tcgen05 products of both; DGXM_ATTN_ONE_CTA runs single CTAs instead.  Held
to the single-CTA kernel's contract: bf16 output max-abs <= 2e-2 and
rel-L2 <= 5e-3 against fp32 attention, LSE within 2e-3; masks, biases, the
fp16 and fp32-output variants and the routed epilogue unchanged.  The shapes
cover odd numbers of 256-row Q blocks (the grid is rounded up to whole pairs,
the spare CTA's rows lying past the queries) and key tails shorter than one
CTA's 64-key half.
"""
from __future__ import annotations

import math

import pytest
import torch

from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, LSE_ABS, SHAPES, reference_attention, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture
def pair(lib):
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ops import set_cta_pair

    set_cta_pair(True)
    try:
        yield
    finally:
        set_cta_pair(True)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def _qkv(shape, seed, dtype=torch.bfloat16):
    b, lq, lk, h, hkv = shape
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(b, lq, h, 128, device="cuda", generator=g).to(dtype)
    k = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).to(dtype)
    v = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).to(dtype)
    return q, k, v


@pytest.mark.parametrize("shape", SHAPES + [(1, 1300, 1090, 2, 1), (1, 256, 40, 1, 1)])
def test_pair_bf16_matches_fp32_reference(pair, shape):
    from dgx_monarch_b200.ops import attention_fwd

    q, k, v = _qkv(shape, 0)
    out, lse = attention_fwd(q, k, v)
    torch.cuda.synchronize()
    ref, ref_lse = reference_attention(q, k, v)
    assert torch.isfinite(out.float()).all()
    assert (out.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS


def test_pair_and_single_cta_agree(lib):
    """The pair's products are the same per-row dot products the single-CTA
    kernel issues, split over two SMs; the outputs agree to within rounding."""
    from dgx_monarch_b200.ops import attention_fwd, set_cta_pair

    q, k, v = _qkv((1, 2048, 2048, 4, 4), 3)
    two, two_lse = attention_fwd(q, k, v)
    set_cta_pair(False)
    try:
        one, one_lse = attention_fwd(q, k, v)
    finally:
        set_cta_pair(True)
    torch.cuda.synchronize()
    assert (one.float() - two.float()).abs().max().item() <= 1e-2
    assert (one_lse - two_lse).abs().max().item() <= 1e-3


def test_pair_fast_and_safe_orders_agree_bitwise(pair):
    from dgx_monarch_b200.ops import attention_fwd

    q, k, v = _qkv((1, 1024, 1536, 2, 2), 1)
    fast, fast_lse = attention_fwd(q, k, v)
    safe, safe_lse = attention_fwd(q, k, v, safe_order=True)
    torch.cuda.synchronize()
    assert torch.equal(fast, safe)
    assert torch.equal(fast_lse, safe_lse)


def test_pair_rescales_a_growing_maximum(pair):
    """Logits that grow block after block force the O rescale in both CTAs."""
    from dgx_monarch_b200.ops import attention_fwd

    g = torch.Generator(device="cuda").manual_seed(9)
    lk = 1024
    q = torch.randn(1, 512, 2, 128, device="cuda", generator=g)
    k = torch.randn(1, lk, 2, 128, device="cuda", generator=g)
    k = k * torch.linspace(0.2, 3.0, lk, device="cuda").view(1, lk, 1, 1)
    v = torch.randn(1, lk, 2, 128, device="cuda", generator=g)
    q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    out, lse = attention_fwd(q, k, v)
    torch.cuda.synchronize()
    ref, ref_lse = reference_attention(q, k, v)
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS


def test_pair_fp16_and_fp32_output_over_strided_inputs(pair):
    from dgx_monarch_b200.ops import attention_fwd

    g = torch.Generator(device="cuda").manual_seed(2)
    qkv = torch.randn(1, 700, 3, 4, 128, device="cuda", generator=g).half()
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    out, lse = attention_fwd(q, k, v, out_dtype=torch.float32, softmax_scale=0.05)
    out16, _ = attention_fwd(q, k, v)
    torch.cuda.synchronize()
    ref, ref_lse = reference_attention(q, k, v, scale=0.05)
    assert out.dtype == torch.float32 and out16.dtype == torch.float16
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS
    ref16, _ = reference_attention(q, k, v)
    assert rel_l2(out16, ref16) <= BF16_REL_L2


def test_pair_keep_masks_and_bias_groups(pair):
    """Pad exclusion and query-group biases run in the softmax of each CTA."""
    from dgx_monarch_b200.ops import attention_fwd_ext, keep_bits

    g = torch.Generator(device="cuda").manual_seed(31)
    rows, heads = 700, 2
    q, k, v = (torch.randn(1, rows, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    drop = [0, 5, 63, 64, 127, 128, 255, 256, 311, 699]
    kk = keep_bits(rows, drop, q.device)
    out, lse = attention_fwd_ext(q, k, v, key_keep=kk, query_keep=kk,
                                 lse=torch.empty(1, heads, rows, device="cuda"))
    keep = [i for i in range(rows) if i not in drop]
    ref, ref_lse = reference_attention(q[:, keep], k[:, keep], v[:, keep])
    assert (out[:, keep].float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert torch.equal(out[:, drop], torch.zeros_like(out[:, drop]))
    assert (lse[:, :, keep] - ref_lse).abs().max().item() <= LSE_ABS

    bias = torch.randn(1, heads, 1, rows, device="cuda", generator=g)
    bias[..., 100:140] = float("-inf")
    groups = [(0, 300, None), (300, rows, bias)]
    out, _ = attention_fwd_ext(q, k, v, bias_groups=groups)
    torch.cuda.synchronize()
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    for start, end, b in groups:
        logits = qf[:, :, start:end] @ kf.transpose(-1, -2) / math.sqrt(128)
        if b is not None:
            logits = logits + b
        want = (torch.softmax(logits, -1) @ vf).transpose(1, 2)
        assert rel_l2(out[:, start:end], want) <= BF16_REL_L2


def test_pair_routed_epilogue_equals_plain_output(pair):
    """The routed epilogue (inverse all-to-all stores) at world 1 writes the
    same bits as the plain output."""
    from dgx_monarch_b200.ops import attention_fwd
    from dgx_monarch_b200.ulysses import attention_routed

    q, k, v = _qkv((1, 1000, 1000, 3, 3), 5)
    plain, _ = attention_fwd(q, k, v)
    routed = torch.empty_like(q)
    attention_routed(q, k, v, [routed.data_ptr()], (1000 * 3 * 128, 3 * 128, 128), world=1, rank=0,
                     seq_local=1000)
    torch.cuda.synchronize()
    assert torch.equal(plain, routed)
