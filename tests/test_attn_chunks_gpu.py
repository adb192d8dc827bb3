"""The release of P in chunks (DGXM_ATTN_P_CHUNKS): the softmax hands each
128-key block's probabilities to the tensor core in 4 chunks (2 for e4m3),
the library default, and the P.V steps of a chunk start while the rest is
computed; one chunk is kept as a cross-check.  Both are held to the same
contract: bf16 output max-abs <= 2e-2 and rel-L2 <= 5e-3, LSE within 2e-3
of fp32 attention; e4m3 rel-L2 <= 3e-2; masks and routing unchanged.
"""
from __future__ import annotations

import pytest
import torch

from tests.test_attn_gpu import (BF16_MAX_ABS, BF16_REL_L2, FP8_REL_L2, LSE_ABS, SHAPES,
                                 quantize_e4m3_per_head, reference_attention, rel_l2)

pytestmark = pytest.mark.gpu


@pytest.fixture
def chunks(request):
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ops import set_p_chunks

    set_p_chunks(request.param)
    try:
        yield request.param
    finally:
        set_p_chunks(0)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("chunks", [1, 4], indirect=True)
@pytest.mark.parametrize("shape", SHAPES)
def test_chunked_bf16_matches_fp32_reference(lib, chunks, shape):
    from dgx_monarch_b200.ops import attention_fwd

    b, lq, lk, h, hkv = shape
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(b, lq, h, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).bfloat16()
    out, lse = attention_fwd(q, k, v)
    torch.cuda.synchronize()
    ref, ref_lse = reference_attention(q, k, v)
    assert torch.isfinite(out.float()).all()
    assert (out.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS


@pytest.mark.parametrize("chunks", [1, 4], indirect=True)
def test_chunked_rescales_a_growing_maximum(lib, chunks):
    """Logits that grow block after block force the O rescale, which the
    chunked kernel performs before releasing a block's first chunk."""
    from dgx_monarch_b200.ops import attention_fwd

    g = torch.Generator(device="cuda").manual_seed(9)
    lk = 1024
    q = torch.randn(1, 256, 2, 128, device="cuda", generator=g)
    k = torch.randn(1, lk, 2, 128, device="cuda", generator=g)
    k *= torch.linspace(0.2, 6.0, lk, device="cuda").view(1, lk, 1, 1)
    v = torch.randn(1, lk, 2, 128, device="cuda", generator=g)
    q, k, v = (x.bfloat16() for x in (q, k, v))
    out, lse = attention_fwd(q, k, v)
    torch.cuda.synchronize()
    ref, ref_lse = reference_attention(q, k, v)
    assert (out.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS


@pytest.mark.parametrize("chunks", [1, 4], indirect=True)
@pytest.mark.parametrize("shape", [(1, 256, 256, 2, 2), (2, 4608, 4608, 3, 3), (1, 1000, 333, 4, 2)])
def test_chunked_fp8_matches_sdpa(lib, chunks, shape):
    from dgx_monarch_b200.ops import attention_fwd

    b, lq, lk, h, hkv = shape
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn(b, n, hh, 128, device="cuda", generator=g).bfloat16()
               for n, hh in ((lq, h), (lk, hkv), (lk, hkv)))
    (q8, qs), (k8, ks), (v8, vs) = (quantize_e4m3_per_head(x) for x in (q, k, v))
    out, lse = attention_fwd(q8, k8, v8, q_descale=qs, k_descale=ks, v_descale=vs)
    torch.cuda.synchronize()
    deq = [x.float() * s.view(1, 1, -1, 1) for x, s in ((q8, qs), (k8, ks), (v8, vs))]
    ref, ref_lse = reference_attention(*deq)
    assert rel_l2(out, ref) <= FP8_REL_L2
    assert (lse - ref_lse).abs().max().item() <= 5 * LSE_ABS


@pytest.mark.parametrize("chunks", [1, 4], indirect=True)
def test_chunked_keep_masks_and_routing(lib, chunks):
    """The extras kernel (keep bits) and the routed epilogue with chunks."""
    from dgx_monarch_b200.ops import attention_fwd_ext, keep_bits

    g = torch.Generator(device="cuda").manual_seed(31)
    rows, world, heads = 700, 2, 3
    q, k, v = (torch.randn(1, rows, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    drop = [0, 5, 127, 128, 255, 256, 311, 699]
    kk = keep_bits(rows, drop, q.device)
    ls = rows // world
    outs = [torch.zeros(1, ls, world * heads, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    for r in range(world):
        attention_fwd_ext(q, k, v, key_keep=kk, query_keep=kk,
                          route={"o_peers": [o.data_ptr() for o in outs], "world": world, "rank": r,
                                 "seq_local": ls},
                          out_strides=(ls * world * heads * 128, world * heads * 128, 128))
    torch.cuda.synchronize()
    keep = [i for i in range(rows) if i not in drop]
    ref, _ = reference_attention(q[:, keep], k[:, keep], v[:, keep])
    got = torch.cat(outs, dim=1)[:, :, :heads]
    assert (got[:, keep].float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(got[:, keep], ref) <= BF16_REL_L2
    assert got[:, drop].abs().max().item() == 0.0


@pytest.mark.parametrize("shape", [(1, 256, 256, 1, 1), (2, 300, 77, 3, 1), (1, 4096, 4096, 2, 2)])
def test_one_and_four_chunks_agree(lib, shape):
    """The chunked release accumulates the P.V steps in another order than the
    single release; the two agree within the bf16 bound, and the LSE (computed
    before any P.V) is the same bits."""
    from dgx_monarch_b200.ops import attention_fwd, set_p_chunks

    b, lq, lk, h, hkv = shape
    g = torch.Generator(device="cuda").manual_seed(17)
    q = torch.randn(b, lq, h, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).bfloat16()
    four, four_lse = attention_fwd(q, k, v)
    set_p_chunks(1)
    try:
        one, one_lse = attention_fwd(q, k, v)
    finally:
        set_p_chunks(0)
    torch.cuda.synchronize()
    assert (four_lse - one_lse).abs().max().item() <= 1e-5
    assert rel_l2(four, one.float()) <= BF16_REL_L2
