"""Parity at the benchmark configurations' real sizes, one GPU each.

The kernels' tile counts, TMA coordinates and 32-bit row arithmetic depend on
the sequence length, so each configuration runs at its own size here, against
a chunked fp32 reference on the device (torch matmul in full fp32):

- Wan video layer: the whole 75,600-token axis, two of the 40 heads, every
  query row, through UlyssesAttention at world 1; and all 40 heads on a
  sample of query rows.
- Flux/Krea2 double block at Ulysses-8: the joint [text | image] layout of
  64 text + 1152 image rows per rank, 24 heads, the 8 ranks emulated on one
  GPU -- the seg0 scatter (the joint order of adapters/usp_sequence_order.py:
  33-146), bit-exact against the oracle, then the routed epilogue.
- CFG + FP8: batch 2 x 4,608 tokens x 24 heads in e4m3 with per-head absmax
  scales, held to 3e-2 against SDPA over the same e4m3 inputs and, against the
  unquantized activations, to the format's own floor plus that 3e-2.
- Long-video hybrid: one ring step (54,900 local query rows x 2 heads against
  one 54,900-row K/V block) and the LSE merge over 4 blocks (219,600 keys).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import usp
from tests.test_attn_gpu import (BF16_MAX_ABS, BF16_REL_L2, FP8_REL_L2, LSE_ABS, reference_attention,
                                 rel_l2)

pytestmark = pytest.mark.gpu


def _randn(shape, g):
    return torch.randn(*shape, device="cuda", generator=g).bfloat16()


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy()


def test_wan_layer_full_axis_two_heads(lib):
    """75,600 tokens (21x90x160 latent, (1,2,2) patches), heads 0-1 of 40."""
    from dgx_monarch_b200.ulysses import UlyssesAttention

    s, heads = 75600, 2
    g = torch.Generator(device="cuda").manual_seed(75600)
    q, k, v = (_randn((1, s, heads, 128), g) for _ in range(3))
    uly = UlyssesAttention(world=1, rank=0, batch=1, seq_local=s, heads=heads, head_dim=128,
                           device=q.device)
    try:
        out = uly.forward(q, k, v)
    finally:
        uly.close()
    torch.cuda.synchronize()
    ref, _ = reference_attention(q, k, v, chunk=1024)
    assert torch.isfinite(out.float()).all()
    assert (out.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(out, ref) <= BF16_REL_L2


def test_wan_layer_all_heads_sampled_rows(lib):
    """All 40 heads of the 75,600-token layer (the benchmark's launch grid),
    checked on 384 query rows spread over the axis, including the last tile's."""
    from dgx_monarch_b200.ops import attention_fwd

    s, heads = 75600, 40
    g = torch.Generator(device="cuda").manual_seed(40)
    q, k, v = (_randn((1, s, heads, 128), g) for _ in range(3))
    out, lse = attention_fwd(q, k, v)
    torch.cuda.synchronize()
    rows = torch.cat((torch.randint(0, s, (320,), device="cuda", generator=g),
                      torch.arange(s - 64, s, device="cuda")))
    ref, ref_lse = reference_attention(q[:, rows], k, v, chunk=128)
    got = out[:, rows]
    assert (got.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(got, ref) <= BF16_REL_L2
    assert (lse[:, :, rows] - ref_lse).abs().max().item() <= LSE_ABS


def test_flux_block_ulysses8_joint_layout(lib):
    """C2 at Ulysses-8: each rank holds [64 text | 1152 image] rows of 24 heads;
    the scatter writes the stock key order bit-exactly, the routed epilogue
    stores exactly what attention + inverse all-to-all store, and the composed
    result is joint attention over the 9,728-row sequence."""
    from dgx_monarch_b200.ops import attention_fwd
    from dgx_monarch_b200.ulysses import attention_routed, ulysses_gather, ulysses_scatter

    world, text, image, heads = 8, 64, 1152, 24
    ls, hl = text + image, heads // world
    s = ls * world
    g = torch.Generator(device="cuda").manual_seed(9728)
    full = [_randn((1, s, heads, 128), g) for _ in range(3)]  # rank-major gathered axis
    local = [[x[:, r * ls:(r + 1) * ls].contiguous() for x in full] for r in range(world)]
    nan = float("nan")
    recv = [[torch.full((1, s, hl, 128), nan, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
            for _ in range(3)]
    for src in range(world):
        ulysses_scatter(local[src], [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)],
                        world=world, rank=src, seg0=text)
    torch.cuda.synchronize()
    order = usp.RankMajorJointOrder(text, image)
    for t in range(3):
        rank_major = usp.seq_all_to_all_4d([_bits(local[r][t]) for r in range(world)], 2, 1)
        for r in range(world):
            canon = order.canonicalize(rank_major[r], rank_major[r], rank_major[r], None, None)[0]
            assert np.array_equal(_bits(recv[t][r]), canon)
    routed = [torch.full((1, ls, heads, 128), nan, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    gathered = [torch.full_like(x, nan) for x in routed]
    strides = (ls * heads * 128, heads * 128, 128)
    for r in range(world):
        attention_routed(recv[0][r], recv[1][r], recv[2][r], [o.data_ptr() for o in routed], strides,
                         world=world, rank=r, seq_local=ls, seg0=text)
        canon_out, _ = attention_fwd(recv[0][r], recv[1][r], recv[2][r], return_lse=False)
        ulysses_gather(canon_out, [o.data_ptr() for o in gathered], world=world, rank=r, seq_local=ls,
                       heads=heads, seg0=text)
    torch.cuda.synchronize()
    for r in range(world):
        assert torch.equal(routed[r], gathered[r])
    ref, _ = reference_attention(*full)
    got = torch.cat(routed, dim=1)
    assert (got.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(got, ref) <= BF16_REL_L2


def test_cfg_fp8_block_both_bounds(lib, record_property):
    """C3: batch 2 (cond/uncond) x (4096 image + 512 text) tokens x 24 heads,
    e4m3 with per-head fp32 absmax scales (amax / 448), bf16 output.

    The configuration fixes the attention inputs as the e4m3 tensors, so the
    3e-2 bound is held against SDPA over those same inputs.  Against SDPA over
    the unquantized bf16 activations the three e4m3 roundings alone (3
    mantissa bits on q, k and v) already move the output; that floor is
    measured here with exact arithmetic on the dequantized inputs, and the
    kernel stays within the floor plus its own 3e-2."""
    from dgx_monarch_b200.ops import attention_fwd
    from dgx_monarch_b200.prologue import quantize_e4m3_per_head

    b, s, heads = 2, 4608, 24
    g = torch.Generator(device="cuda").manual_seed(4608)
    q, k, v = (_randn((b, s, heads, 128), g) for _ in range(3))
    (q8, qs), (k8, ks), (v8, vs) = (quantize_e4m3_per_head(x) for x in (q, k, v))
    out, lse = attention_fwd(q8, k8, v8, q_descale=qs, k_descale=ks, v_descale=vs)
    torch.cuda.synchronize()
    deq = [x.float() * sc.view(1, 1, -1, 1) for x, sc in ((q8, qs), (k8, ks), (v8, vs))]
    ref_deq, ref_deq_lse = reference_attention(*deq)
    ref_act, _ = reference_attention(q, k, v)
    vs_inputs = rel_l2(out, ref_deq)
    vs_activations = rel_l2(out, ref_act)
    floor = rel_l2(ref_deq, ref_act)
    record_property("fp8_rel_l2_vs_sdpa_of_e4m3_inputs", vs_inputs)
    record_property("fp8_rel_l2_vs_sdpa_of_activations", vs_activations)
    record_property("e4m3_input_floor_vs_activations", floor)
    print(f"C3 e4m3: rel-L2 {vs_inputs:.4f} vs SDPA(e4m3 inputs), {vs_activations:.4f} vs "
          f"SDPA(activations); input-format floor {floor:.4f}")
    assert torch.isfinite(out.float()).all()
    assert vs_inputs <= FP8_REL_L2
    assert (lse - ref_deq_lse).abs().max().item() <= 5 * LSE_ABS
    assert vs_activations <= floor + FP8_REL_L2


def test_long_video_ring_step_and_merge(lib):
    """C5 (Ulysses-2 x ring-4 over 219,600 tokens, 24 heads): each rank holds
    54,900 query rows of 12 heads and attends four 54,900-row K/V blocks.
    Two of the heads: one ring step against its fp32 reference (out and LSE),
    then the merge of all four steps against attention over every key."""
    from dgx_monarch_b200.ops import attention_fwd, lse_merge

    rows, blocks, heads = 54900, 4, 2
    g = torch.Generator(device="cuda").manual_seed(219600)
    q = _randn((1, rows, heads, 128), g)
    k, v = (_randn((1, rows * blocks, heads, 128), g) for _ in range(2))
    blk = lambda t, i: t[:, i * rows:(i + 1) * rows]
    parts = [attention_fwd(q, blk(k, i), blk(v, i), out_dtype=torch.float32) for i in range(blocks)]
    torch.cuda.synchronize()
    step_ref, step_lse = reference_attention(q, blk(k, 0), blk(v, 0), chunk=1024)
    assert rel_l2(parts[0][0], step_ref) <= BF16_REL_L2
    assert (parts[0][0] - step_ref).abs().max().item() <= BF16_MAX_ABS
    assert (parts[0][1] - step_lse).abs().max().item() <= LSE_ABS
    del step_ref, step_lse
    out, lse = lse_merge([p[0] for p in parts], [p[1] for p in parts])
    torch.cuda.synchronize()
    ref, ref_lse = reference_attention(q, k, v, chunk=512)
    assert (out.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS
