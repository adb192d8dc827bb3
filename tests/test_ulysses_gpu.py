"""Ulysses all-to-all kernels against the oracle, ranks emulated on one GPU.

Every emulated rank's receive tensors live on the same device; each source
rank's scatter is its own launch and no kernel waits on another, so the
emulation needs no cross-launch synchronisation.  Layout results are
bit-exact against oracle.usp.seq_all_to_all_4d (the rank-major convention the
reference pins in tests/test_usp_full_axis.py); attention results within the
bf16 tolerance of an fp32 reference.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import usp
from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, reference_attention, rel_l2

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy()


@pytest.mark.parametrize("world,batch,seq_local,heads", [(2, 1, 64, 4), (4, 2, 33, 8), (8, 1, 17, 40)])
def test_scatter_is_bit_exact_rank_major(lib, world, batch, seq_local, heads):
    from dgx_monarch_b200.ulysses import ulysses_scatter

    g = torch.Generator(device="cuda").manual_seed(world)
    local = [[torch.randn(batch, seq_local, heads, 128, device="cuda", generator=g).bfloat16()
              for _ in range(3)] for _ in range(world)]
    hl = heads // world
    recv = [[torch.full((batch, seq_local * world, hl, 128), float("nan"), device="cuda",
                        dtype=torch.bfloat16) for _ in range(world)] for _ in range(3)]
    for src in range(world):
        ulysses_scatter(local[src], [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)],
                        world=world, rank=src)
    torch.cuda.synchronize()
    for t in range(3):
        want = usp.seq_all_to_all_4d([_bits(local[s][t]) for s in range(world)], 2, 1)
        for r in range(world):
            assert np.array_equal(_bits(recv[t][r]), want[r])


@pytest.mark.parametrize("world,batch,seq_local,heads", [(2, 1, 64, 4), (4, 2, 33, 8), (8, 1, 17, 40)])
def test_copy_engine_scatter_is_bit_exact_rank_major(lib, world, batch, seq_local, heads):
    """The copy-engine scatter (strided 2-D copies per tensor and destination)
    writes the same bytes as the kernel, including from a head-group slice."""
    from dgx_monarch_b200.ulysses import ulysses_scatter_copy

    g = torch.Generator(device="cuda").manual_seed(world + 50)
    wide = [[torch.randn(batch, seq_local, 2 * heads, 128, device="cuda", generator=g).bfloat16()
             for _ in range(3)] for _ in range(world)]
    local = [[t[:, :, heads:] for t in ts] for ts in wide]  # a group's head slice: strided rows
    hl = heads // world
    recv = [[torch.full((batch, seq_local * world, hl, 128), float("nan"), device="cuda",
                        dtype=torch.bfloat16) for _ in range(world)] for _ in range(3)]
    for src in range(world):
        ulysses_scatter_copy(local[src], [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)],
                             world=world, rank=src)
    torch.cuda.synchronize()
    for t in range(3):
        want = usp.seq_all_to_all_4d([_bits(local[s][t]) for s in range(world)], 2, 1)
        for r in range(world):
            assert np.array_equal(_bits(recv[t][r]), want[r])


def test_scatter_reads_strided_projection_views(lib):
    """q/k/v as views of one packed (B, L, 3, H, D) projection output."""
    from dgx_monarch_b200.ulysses import ulysses_scatter

    world, heads, ls = 2, 4, 40
    g = torch.Generator(device="cuda").manual_seed(5)
    packed = [torch.randn(1, ls, 3, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(world)]
    recv = [[torch.zeros(1, ls * world, heads // world, 128, device="cuda", dtype=torch.bfloat16)
             for _ in range(world)] for _ in range(3)]
    for src in range(world):
        views = [packed[src][:, :, i] for i in range(3)]
        ulysses_scatter(views, [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)],
                        world=world, rank=src)
    torch.cuda.synchronize()
    for t in range(3):
        want = usp.seq_all_to_all_4d([_bits(packed[s][:, :, t]) for s in range(world)], 2, 1)
        for r in range(world):
            assert np.array_equal(_bits(recv[t][r]), want[r])


@pytest.mark.parametrize("world,seq_local,heads", [(2, 96, 4), (4, 50, 8)])
def test_gather_is_bit_exact_inverse(lib, world, seq_local, heads):
    from dgx_monarch_b200.ulysses import ulysses_gather

    g = torch.Generator(device="cuda").manual_seed(11)
    hl = heads // world
    full = [torch.randn(1, seq_local * world, hl, 128, device="cuda", generator=g).bfloat16()
            for _ in range(world)]
    outs = [torch.zeros(1, seq_local, heads, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    for src in range(world):
        ulysses_gather(full[src], [o.data_ptr() for o in outs], world=world, rank=src,
                       seq_local=seq_local, heads=heads)
    torch.cuda.synchronize()
    want = usp.seq_all_to_all_4d([_bits(f) for f in full], 1, 2)
    for r in range(world):
        assert np.array_equal(_bits(outs[r]), want[r])


@pytest.mark.parametrize("world,seq_local,heads", [(2, 300, 4), (4, 257, 8)])
def test_routed_epilogue_equals_attention_then_gather(lib, world, seq_local, heads):
    """The fused inverse all-to-all stores exactly what attention + gather store,
    and the composed Ulysses result matches unsharded attention."""
    from dgx_monarch_b200.ops import attention_fwd
    from dgx_monarch_b200.ulysses import attention_routed, ulysses_gather, ulysses_scatter

    g = torch.Generator(device="cuda").manual_seed(13)
    s = seq_local * world
    hl = heads // world
    q, k, v = (torch.randn(1, s, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    local = [[x[:, r * seq_local:(r + 1) * seq_local].contiguous() for x in (q, k, v)] for r in range(world)]
    recv = [[torch.empty(1, s, hl, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
            for _ in range(3)]
    for src in range(world):
        ulysses_scatter(local[src], [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)],
                        world=world, rank=src)
    routed = [torch.zeros(1, seq_local, heads, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    gathered = [torch.zeros_like(x) for x in routed]
    strides = (seq_local * heads * 128, heads * 128, 128)
    for r in range(world):
        attention_routed(recv[0][r], recv[1][r], recv[2][r], [o.data_ptr() for o in routed], strides,
                         world=world, rank=r, seq_local=seq_local)
        full_out, _ = attention_fwd(recv[0][r], recv[1][r], recv[2][r])
        ulysses_gather(full_out, [o.data_ptr() for o in gathered], world=world, rank=r,
                       seq_local=seq_local, heads=heads)
    torch.cuda.synchronize()
    for r in range(world):
        assert torch.equal(routed[r], gathered[r])
    ref, _ = reference_attention(q, k, v)
    got = torch.cat(routed, dim=1)
    assert (got.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(got, ref) <= BF16_REL_L2


@pytest.mark.parametrize("world,text,image,heads", [(2, 3, 5, 4), (4, 16, 48, 8), (8, 64, 1152 // 8, 24)])
def test_joint_order_scatter_is_canonical_bit_exact(lib, world, text, image, heads):
    """seg0 > 0 writes the stock [t0,t1,...,i0,i1,...] order that
    RankMajorJointOrder.canonicalize (adapters/usp_sequence_order.py:105-146)
    produces from the rank-major gathered axis."""
    from dgx_monarch_b200.ulysses import ulysses_gather, ulysses_scatter

    g = torch.Generator(device="cuda").manual_seed(17)
    ls = text + image
    local = [torch.randn(1, ls, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(world)]
    hl = heads // world
    recv = [torch.zeros(1, ls * world, hl, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    for src in range(world):
        ulysses_scatter([local[src]], [[recv[r].data_ptr() for r in range(world)]], world=world,
                        rank=src, seg0=text)
    torch.cuda.synchronize()
    rank_major = usp.seq_all_to_all_4d([_bits(t) for t in local], 2, 1)
    order = usp.RankMajorJointOrder(text, image)
    for r in range(world):
        canon, _, _, _, _, _ = order.canonicalize(rank_major[r], rank_major[r], rank_major[r], None, None)
        assert np.array_equal(_bits(recv[r]), canon)
    # The inverse with the same row map returns every rank's own rows.
    back = [torch.zeros_like(x) for x in local]
    for src in range(world):
        ulysses_gather(recv[src], [b.data_ptr() for b in back], world=world, rank=src,
                       seq_local=ls, heads=heads, seg0=text)
    torch.cuda.synchronize()
    for r in range(world):
        assert torch.equal(back[r], local[r])


def test_joint_order_routed_epilogue_matches_gather(lib):
    from dgx_monarch_b200.ops import attention_fwd
    from dgx_monarch_b200.ulysses import attention_routed, ulysses_gather, ulysses_scatter

    world, text, image, heads = 2, 64, 192, 4
    ls = text + image
    g = torch.Generator(device="cuda").manual_seed(19)
    local = [[torch.randn(1, ls, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3)]
             for _ in range(world)]
    hl = heads // world
    recv = [[torch.empty(1, ls * world, hl, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
            for _ in range(3)]
    for src in range(world):
        ulysses_scatter(local[src], [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)],
                        world=world, rank=src, seg0=text)
    routed = [torch.zeros(1, ls, heads, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    gathered = [torch.zeros_like(x) for x in routed]
    for r in range(world):
        attention_routed(recv[0][r], recv[1][r], recv[2][r], [o.data_ptr() for o in routed],
                         (ls * heads * 128, heads * 128, 128), world=world, rank=r, seq_local=ls, seg0=text)
        full, _ = attention_fwd(recv[0][r], recv[1][r], recv[2][r])
        ulysses_gather(full, [o.data_ptr() for o in gathered], world=world, rank=r, seq_local=ls,
                       heads=heads, seg0=text)
    torch.cuda.synchronize()
    for r in range(world):
        assert torch.equal(routed[r], gathered[r])
    # And the composition is joint attention over the whole [text, image] sequence.
    q, k, v = (torch.cat([local[r][t] for r in range(world)], dim=1) for t in range(3))
    ref, _ = reference_attention(q, k, v)
    got = torch.cat(routed, dim=1)
    assert rel_l2(got, ref) <= BF16_REL_L2


def test_emulated_ring_merge_equals_full_attention(lib):
    """Ring order of oracle.usp.ring_attention on one GPU: rank r attends the
    block of rank (r - t) mod R at step t; the LSE merge of the R partial
    results equals attention over the whole key axis."""
    from dgx_monarch_b200.ops import attention_fwd, lse_merge

    world, rows = 4, 300
    g = torch.Generator(device="cuda").manual_seed(23)
    q, k, v = (torch.randn(1, rows * world, 3, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    blk = lambda t, r: t[:, r * rows:(r + 1) * rows].contiguous()
    ref, ref_lse = reference_attention(q, k, v)
    for r in range(world):
        parts = [attention_fwd(blk(q, r), blk(k, (r - t) % world), blk(v, (r - t) % world),
                               out_dtype=torch.float32) for t in range(world)]
        out, lse = lse_merge([p[0] for p in parts], [p[1] for p in parts])
        torch.cuda.synchronize()
        assert rel_l2(out, ref[:, r * rows:(r + 1) * rows]) <= BF16_REL_L2
        assert (lse - ref_lse[:, :, r * rows:(r + 1) * rows]).abs().max().item() <= 2e-3


@pytest.mark.parametrize("world,batch,image_local,text,heads,text_first", [
    (2, 1, 512, 256, 8, True),     # 1024 image + 256 text rows, 8 heads, split 2-way
    (4, 2, 75, 77, 8, False),      # ragged tiles, text after the image
    (8, 1, 40, 13, 16, True),
    (1, 1, 300, 33, 4, True)])
def test_replicated_text_joint_emulated_ranks(lib, world, batch, image_local, text, heads, text_first):
    """Joint attention with the image split by sequence and the text replicated.

    - Every receive tensor holds this rank's head slice of the text next to the
      rank-major image rows (bit-exact).
    - The routed epilogue stores exactly what per-rank attention over the
      receive tensor computes: image rows at their owners, text rows at every
      rank (bit-exact), so all ranks hold the same text output.
    - The result matches one-process attention over the unsharded concatenation.
    """
    from dgx_monarch_b200.ops import attention_fwd, attention_fwd_ext
    from dgx_monarch_b200.ulysses import ulysses_scatter_joint

    g = torch.Generator(device="cuda").manual_seed(100 + world)
    ls, hl, d = image_local, heads // world, 128
    s_img = ls * world
    rows = text + s_img
    img = [torch.randn(batch, s_img, heads, d, device="cuda", generator=g).bfloat16() for _ in range(3)]
    txt = [torch.randn(batch, text, heads, d, device="cuda", generator=g).bfloat16() for _ in range(3)]
    nan = float("nan")
    recv = [[torch.full((batch, rows, hl, d), nan, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
            for _ in range(3)]
    for src in range(world):
        local = [x[:, src * ls:(src + 1) * ls].contiguous() for x in img]
        ulysses_scatter_joint(local, txt, [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)],
                              world=world, rank=src, text_first=text_first)
    torch.cuda.synchronize()
    for t in range(3):
        for r in range(world):
            heads_r = slice(r * hl, (r + 1) * hl)
            parts = [txt[t][:, :, heads_r], img[t][:, :, heads_r]]
            want = torch.cat(parts if text_first else parts[::-1], dim=1)
            assert torch.equal(recv[t][r], want)

    img_out = [torch.full((batch, ls, heads, d), nan, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    txt_out = [torch.full((batch, text, heads, d), nan, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    for r in range(world):
        attention_fwd_ext(recv[0][r], recv[1][r], recv[2][r],
                          route={"o_peers": [o.data_ptr() for o in img_out], "world": world, "rank": r,
                                 "seq_local": ls, "txt_rows": text, "txt_front": text_first,
                                 "txt_peers": [o.data_ptr() for o in txt_out]},
                          out_strides=(ls * heads * d, heads * d, d))
    torch.cuda.synchronize()
    for r in range(world):
        full, _ = attention_fwd(recv[0][r], recv[1][r], recv[2][r], return_lse=False)
        f_txt, f_img = (full[:, :text], full[:, text:]) if text_first else (full[:, s_img:], full[:, :s_img])
        heads_r = slice(r * hl, (r + 1) * hl)
        for owner in range(world):
            assert torch.equal(img_out[owner][:, :, heads_r], f_img[:, owner * ls:(owner + 1) * ls])
            assert torch.equal(txt_out[owner][:, :, heads_r], f_txt)
    q, k, v = (torch.cat([a, b] if text_first else [b, a], dim=1) for a, b in zip(txt, img))
    ref, _ = reference_attention(q, k, v)
    ref_txt, ref_img = (ref[:, :text], ref[:, text:]) if text_first else (ref[:, s_img:], ref[:, :s_img])
    got_img = torch.cat(img_out, dim=1)
    for got, want in ((got_img, ref_img), (txt_out[0], ref_txt)):
        assert (got.float() - want).abs().max().item() <= BF16_MAX_ABS
        assert rel_l2(got, want) <= BF16_REL_L2


@pytest.mark.parametrize("head_dim,dtype,text_first", [
    (64, torch.float32, True),     # the fp32, head_dim 64 CPU/gloo joint case's data
    (64, torch.float32, False),
    (96, torch.float16, True),
    (128, torch.bfloat16, True)])
def test_joint_ulysses_class_one_rank(lib, head_dim, dtype, text_first, record_property):
    """JointUlyssesAttention on one rank: any float dtype in and out (bf16
    compute), head_dim below 128 zero-padded with the softmax scale of the real
    head_dim; 1024 image + 256 text rows, 8 heads."""
    from dgx_monarch_b200.ulysses import JointUlyssesAttention

    dev = torch.device("cuda")
    g = torch.Generator(device="cuda").manual_seed(head_dim)
    img = [torch.randn(1, 1024, 8, head_dim, device=dev, generator=g).to(dtype) for _ in range(3)]
    txt = [torch.randn(1, 256, 8, head_dim, device=dev, generator=g).to(dtype) for _ in range(3)]
    joint = JointUlyssesAttention(world=1, rank=0, batch=1, seq_local=1024, txt_rows=256, heads=8,
                                  head_dim=head_dim, device=dev, text_first=text_first)
    try:
        out_img, out_txt = joint(*img, *txt)
        again_img, again_txt = joint(*img, *txt)
    finally:
        joint.close()
    assert out_img.dtype == dtype and out_txt.dtype == dtype
    assert out_img.shape == (1, 1024, 8, head_dim) and out_txt.shape == (1, 256, 8, head_dim)
    assert torch.equal(out_img, again_img) and torch.equal(out_txt, again_txt)
    # Held against fp32 attention over the caller's own (unrounded) inputs:
    # the bf16 compute, the rounding of fp32 inputs to it included, stays
    # within the bf16 bounds.
    q, k, v = (torch.cat([a, b] if text_first else [b, a], dim=1).float() for a, b in zip(txt, img))
    ref, _ = reference_attention(q, k, v)
    ref_txt, ref_img = (ref[:, :256], ref[:, 256:]) if text_first else (ref[:, 1024:], ref[:, :1024])
    for got, want in ((out_img, ref_img), (out_txt, ref_txt)):
        assert (got.float() - want).abs().max().item() <= BF16_MAX_ABS
        assert rel_l2(got, want) <= BF16_REL_L2
    record_property("rel_l2_vs_fp32_of_unrounded_inputs",
                    max(rel_l2(out_img, ref_img), rel_l2(out_txt, ref_txt)))


def test_joint_ulysses_without_text_is_plain_attention(lib):
    """No text rows: the joint step is bit-identical to the attention kernel."""
    from dgx_monarch_b200.ops import attention_fwd
    from dgx_monarch_b200.ulysses import JointUlyssesAttention

    dev = torch.device("cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn(2, 200, 4, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    joint = JointUlyssesAttention(world=1, rank=0, batch=2, seq_local=200, txt_rows=0, heads=4, head_dim=128,
                                  device=dev)
    empty = torch.empty(2, 0, 4, 128, device=dev, dtype=torch.bfloat16)
    try:
        out, out_txt = joint(q, k, v, empty, empty, empty)
    finally:
        joint.close()
    want, _ = attention_fwd(q, k, v, return_lse=False)
    assert out_txt.shape == (2, 0, 4, 128)
    assert torch.equal(out, want)
