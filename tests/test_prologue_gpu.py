"""Fused Q/K norm + RoPE + Ulysses scatter, and per-head e4m3 quantisation.

The prologue is checked against the separate ops it replaces, composed in
torch with the same rounding points (norm output rounded to bf16, weight
product rounded, RoPE in fp32 then rounded), and its layout against the
oracle's all-to-all: values within one bf16 ulp (the norm's sum order and
rsqrt differ), V bit-exact.  Quantisation is bit-exact against torch.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import usp

pytestmark = pytest.mark.gpu


def _ref_norm_rope(x, w, mode, eps, table):
    """The unfused composition in torch: (B, L, H, D) bf16 -> bf16."""
    xf = x.float()
    b, l, h, d = x.shape
    if mode == "hidden":
        flat = xf.reshape(b, l, h * d)
        sc = torch.rsqrt(flat.pow(2).mean(-1, keepdim=True) + eps)
        n = (flat * sc).bfloat16()
        n = (n.float() * w.float()).bfloat16().reshape(b, l, h, d)
    elif mode == "head":
        sc = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        n = (xf * sc).bfloat16()
        n = (n.float() * w.float()).bfloat16()
    else:
        n = x
    if table is None:
        return n
    nf = n.float()
    c = table[..., 0][None, :, None, :]
    s = table[..., 1][None, :, None, :]
    x0, x1 = nf[..., 0::2], nf[..., 1::2]
    out = torch.empty_like(nf)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out.bfloat16()


def _within_one_ulp(got, want):
    g, w = got.float(), want.float()
    tol = 2.0 ** -7 * torch.maximum(g.abs(), w.abs()) + 1e-6
    return bool(((g - w).abs() <= tol).all())


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy()


@pytest.mark.parametrize("mode,world,heads,axes", [
    ("hidden", 4, 40, [44, 42, 42]),   # Wan: norm over 5120, 3-axis RoPE
    ("head", 2, 24, [16, 56, 56]),     # Flux/Krea2: per-head QKNorm, axis 0 unused by images
    ("none", 2, 8, None),
    ("head", 1, 5, [16, 56, 56]),      # an odd head count: a warp's halves straddle the k / v rows
    ("head", 3, 9, [16, 56, 56]),
])
def test_prologue_matches_unfused_ops(lib, mode, world, heads, axes):
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.prologue import qkv_prologue_scatter, rope_table

    ls, eps = 90, 1e-6
    g = torch.Generator(device="cuda").manual_seed(29)
    # q/k/v as views of one packed projection output (B, Ls, 3, H, D).
    packed = [torch.randn(1, ls, 3, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(world)]
    wdim = heads * 128 if mode == "hidden" else 128
    wq = (1 + 0.1 * torch.randn(wdim, device="cuda", generator=g)).bfloat16()
    wk = (1 + 0.1 * torch.randn(wdim, device="cuda", generator=g)).bfloat16()
    tables = [None] * world
    if axes is not None:
        for r in range(world):
            rows = torch.arange(r * ls, (r + 1) * ls, device="cuda")
            pos = torch.stack((rows // 100, (rows // 10) % 10, rows % 10), dim=1)
            tables[r] = rope_table(pos, axes)
    hl = heads // world
    recv = [[torch.zeros(1, ls * world, hl, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
            for _ in range(3)]
    nmode = {"hidden": _lib.NORM_HIDDEN, "head": _lib.NORM_HEAD, "none": _lib.NORM_NONE}[mode]
    for src in range(world):
        q, k, v = (packed[src][:, :, i] for i in range(3))
        qkv_prologue_scatter(q, k, v, [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)],
                             world=world, rank=src, norm_mode=nmode,
                             norm_q_w=wq if mode != "none" else None,
                             norm_k_w=wk if mode != "none" else None, eps=eps, rope=tables[src])
    torch.cuda.synchronize()
    for t, w in ((0, wq), (1, wk), (2, None)):
        want_local = []
        for src in range(world):
            x = packed[src][:, :, t]
            if t < 2:
                x = _ref_norm_rope(x, w, mode, eps, tables[src])
            want_local.append(x.contiguous())
        want = usp.seq_all_to_all_4d([x.float().cpu().numpy() for x in want_local], 2, 1)
        for r in range(world):
            got = recv[t][r]
            if t == 2:
                want_bits = usp.seq_all_to_all_4d([_bits(x) for x in want_local], 2, 1)[r]
                assert np.array_equal(_bits(got), want_bits)
            else:
                assert _within_one_ulp(got, torch.from_numpy(want[r]).cuda())


def test_prologue_joint_order_matches_canonical_layout(lib):
    from dgx_monarch_b200.prologue import qkv_prologue_scatter

    world, text, image, heads = 2, 8, 24, 4
    ls = text + image
    g = torch.Generator(device="cuda").manual_seed(37)
    local = [[torch.randn(1, ls, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3)]
             for _ in range(world)]
    recv = [[torch.zeros(1, ls * world, heads // world, 128, device="cuda", dtype=torch.bfloat16)
             for _ in range(world)] for _ in range(3)]
    for src in range(world):
        qkv_prologue_scatter(*local[src], [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)],
                             world=world, rank=src, seg0=text)
    torch.cuda.synchronize()
    order = usp.RankMajorJointOrder(text, image)
    for t in range(3):
        rank_major = usp.seq_all_to_all_4d([_bits(local[s][t]) for s in range(world)], 2, 1)
        for r in range(world):
            canon = order.canonicalize(rank_major[r], rank_major[r], rank_major[r], None, None)[0]
            assert np.array_equal(_bits(recv[t][r]), canon)


@pytest.mark.parametrize("shape", [(1, 333, 3), (2, 4608, 24)])
def test_quantize_is_bit_exact_against_torch(lib, shape):
    from dgx_monarch_b200.prologue import quantize_e4m3_per_head

    b, l, h = shape
    g = torch.Generator(device="cuda").manual_seed(41)
    x = torch.randn(b, l, h, 128, device="cuda", generator=g).bfloat16()
    q8, descale = quantize_e4m3_per_head(x)
    torch.cuda.synchronize()
    amax = x.float().abs().amax(dim=(0, 1, 3))
    # IEEE division by a tensor (torch divides by a Python scalar through its
    # reciprocal, which rounds differently).
    want_scale = amax / torch.full_like(amax, 448.0)
    want = (x.float() / want_scale.view(1, 1, -1, 1)).to(torch.float8_e4m3fn)
    assert torch.equal(descale, want_scale)
    assert torch.equal(q8.view(torch.uint8), want.view(torch.uint8))


@pytest.mark.parametrize("shape,drop,per_batch", [
    ((1, 333, 3), [7, 40, 331, 332], False),     # scattered pads and a tail
    ((2, 4608, 24), list(range(4600, 4608)), False),
    ((2, 96, 2), None, True),                    # one mask per batch row, one row all pads
])
def test_quantize_with_keep_bits_skips_pad_rows(lib, shape, drop, per_batch):
    """Rows whose keep bit is clear do not set their head's scale: the
    scale is the absmax over the kept rows / 448, and every row (pads
    included, saturated) is written with it."""
    from dgx_monarch_b200.ops import keep_bits
    from dgx_monarch_b200.prologue import quantize_e4m3_per_head

    b, l, h = shape
    g = torch.Generator(device="cuda").manual_seed(l)
    x = torch.randn(b, l, h, 128, device="cuda", generator=g).bfloat16()
    if per_batch:
        keep = torch.stack([keep_bits(l, list(range(0, l, 3)), x.device), keep_bits(l, list(range(l)), x.device)])
        kept = torch.ones(b, l, dtype=torch.bool, device="cuda")
        kept[0, 0::3] = False
        kept[1] = False
    else:
        keep = keep_bits(l, drop, x.device)
        kept = torch.ones(b, l, dtype=torch.bool, device="cuda")
        kept[:, drop] = False
    x[~kept] = x[~kept] * 50  # pads far above the real rows' range
    q8, descale = quantize_e4m3_per_head(x, keep=keep)
    torch.cuda.synchronize()
    amax = (x.float().abs() * kept.view(b, l, 1, 1)).amax(dim=(0, 1, 3)).clamp_min(1e-12)
    want_scale = amax / torch.full_like(amax, 448.0)
    want = (x.float() / want_scale.view(1, 1, -1, 1)).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(descale, want_scale)
    assert torch.equal(q8.view(torch.uint8), want.view(torch.uint8))


def test_batched_quantisation_equals_one_tensor_at_a_time(lib):
    """q, k and v of different rows and head counts (GQA), pads on k and v,
    quantised by one batch of launches: every byte and descale equals the
    one-tensor calls."""
    from dgx_monarch_b200.ops import keep_bits
    from dgx_monarch_b200.prologue import quantize_e4m3_per_head, quantize_e4m3_per_head_many

    g = torch.Generator(device="cuda").manual_seed(303)
    q = torch.randn(2, 700, 6, 128, device="cuda", generator=g).bfloat16()
    k, v = (torch.randn(2, 333, 2, 128, device="cuda", generator=g).bfloat16() for _ in range(2))
    keep = keep_bits(333, [0, 100, 332], q.device)
    got = quantize_e4m3_per_head_many([(q, None, None, None), (k, None, None, keep), (v, None, None, keep)])
    want = [quantize_e4m3_per_head(q), quantize_e4m3_per_head(k, keep=keep), quantize_e4m3_per_head(v, keep=keep)]
    torch.cuda.synchronize()
    for (g8, gs), (w8, ws) in zip(got, want):
        assert torch.equal(gs, ws)
        assert torch.equal(g8.view(torch.uint8), w8.view(torch.uint8))


def _within_ulps(got, want, ulps):
    g, w = got.float(), want.float()
    tol = ulps * 2.0 ** -7 * torch.maximum(g.abs(), w.abs()) + 1e-5
    return ((g - w).abs() > tol).float().mean().item()


@pytest.mark.parametrize("hidden,heads,t_loc,i_loc,rope,bias", [
    (512, 4, 40, 300, True, True),       # tails below and above one 256-row pair tile (odd CTA idle)
    (3072, 24, 64, 300, True, False),    # the C2 block width: 72 pair tiles, 48-step K over a 5-stage ring
    (512, 4, 0, 129, False, True),       # image stream only, no RoPE, one row in the odd CTA
    (1024, 8, 100, 4000, True, True),    # 192 pair tiles: every pair alternates its two accumulators
    (200, 2, 10, 70, True, True),        # K tail (200 = 3 x 64 + 8, zero-filled) and one pair tile of 2 heads
])
def test_fused_qkv_gemm_prologue_matches_separate_ops(lib, hidden, heads, t_loc, i_loc, rope, bias):
    """The QKV Linear + per-head QKNorm + RoPE + sequence->head scatter in one
    tcgen05 kernel, against the separate ops in torch (fp32 GEMM rounded to
    bf16, then the unfused norm / RoPE) and the oracle's all-to-all layout,
    two ranks emulated on one GPU in the joint [text, image] order.  The GEMM
    sums in a different order from torch, so a value may land one bf16 ulp
    away; the fraction of such values is bounded, V's rows differ only there."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.prologue import qkv_gemm_prologue_scatter, rope_table

    world, eps = 2, 1e-6
    ls = t_loc + i_loc
    g = torch.Generator(device="cuda").manual_seed(51)
    w = lambda *shape, s=0.02: (s * torch.randn(*shape, device="cuda", generator=g)).bfloat16()
    n = 3 * heads * 128
    w_txt, w_img = w(n, hidden), w(n, hidden)
    b_txt = w(n, s=0.5) if bias else None
    b_img = w(n, s=0.5) if bias else None
    nq_t, nk_t, nq_i, nk_i = ((1 + w(128, s=0.1)).contiguous() for _ in range(4))
    xs = [(w(t_loc, hidden, s=1.0), w(i_loc, hidden, s=1.0)) for _ in range(world)]
    tables = []
    for r in range(world):
        rows = torch.arange(r * ls, (r + 1) * ls, device="cuda")
        pos = torch.stack((rows // 100, (rows // 10) % 10, rows % 10), dim=1)
        tables.append(rope_table(pos, [16, 56, 56]) if rope else None)
    hl = heads // world
    recv = [[torch.zeros(world * ls, hl, 128, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
            for _ in range(3)]
    ptrs = [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)]
    for r in range(world):
        x_t, x_i = xs[r]
        for x, wq, bb, row0, nq, nk in ((x_t, w_txt, b_txt, 0, nq_t, nk_t), (x_i, w_img, b_img, t_loc, nq_i, nk_i)):
            if x.shape[0] == 0:
                continue
            qkv_gemm_prologue_scatter(x, wq, ptrs, world=world, rank=r, seq_local=ls, row0=row0, seg0=t_loc,
                                      bias=bb, norm_mode=_lib.NORM_HEAD, norm_q_w=nq, norm_k_w=nk, eps=eps,
                                      rope=tables[r])
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    # The separate ops: Linear per stream (fp32 sum, bf16 output), then norm + RoPE.
    want_local = [[None] * world for _ in range(3)]
    for r in range(world):
        x_t, x_i = xs[r]
        parts = []
        for x, wq, bb, nq, nk in ((x_t, w_txt, b_txt, nq_t, nk_t), (x_i, w_img, b_img, nq_i, nk_i)):
            y = x.double() @ wq.double().T
            if bb is not None:
                y = y + bb.double()
            y = y.float().bfloat16().reshape(1, x.shape[0], 3, heads, 128)
            parts.append((y, nq, nk))
        for t in range(3):
            rows = []
            for y, nq, nk in parts:
                tab = None
                if tables[r] is not None:
                    tab = tables[r][:t_loc] if y is parts[0][0] and t_loc else tables[r][t_loc:]
                v = y[:, :, t]
                rows.append(_ref_norm_rope(v, (nq, nk)[t], "head", eps, tab) if t < 2 else v)
            want_local[t][r] = torch.cat(rows, dim=1)
    order = usp.RankMajorJointOrder(t_loc, i_loc)
    for t in range(3):
        # Stock order on the gathered axis: every rank's text rows, then every rank's image rows.
        gathered = [x[0].float().cpu().numpy() for x in want_local[t]]
        full = np.concatenate([np.concatenate([g_[:t_loc] for g_ in gathered]),
                               np.concatenate([g_[t_loc:] for g_ in gathered])])
        for r in range(world):
            want = torch.from_numpy(full[:, r * hl:(r + 1) * hl]).cuda()
            frac = _within_ulps(recv[t][r], want, 2 if t < 2 else 1)
            assert frac <= 2e-3, f"tensor {t} rank {r}: {frac:.2e} of values beyond the ulp bound"
            # No value is further off than two ulps of the largest magnitude.
            diff = (recv[t][r].float() - want).abs().max().item()
            assert diff <= 2.0 ** -6 * want.abs().max().item() + 1e-3, f"tensor {t} rank {r}: max-abs {diff}"
    assert order.text_rows == t_loc


@pytest.mark.parametrize("t_loc,i_loc", [(64, 700), (0, 300), (128, 256)])
def test_grouped_streams_equal_one_call_per_stream(lib, t_loc, i_loc):
    """dgxm_qkv_gemm_prologue_scatter_streams runs a joint block's text and
    image projections (their own weights, biases and QKNorm weights) in one
    launch; every receive row must hold exactly the bits one single-stream
    call per stream writes -- the same tile arithmetic, only the grid is
    shared.  Two ranks emulated on one GPU, joint order, an empty stream."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.prologue import (qkv_gemm_prologue_scatter, qkv_gemm_prologue_scatter_streams,
                                           rope_table)

    world, heads, hidden, eps = 2, 8, 1024, 1e-6
    ls = t_loc + i_loc
    g = torch.Generator(device="cuda").manual_seed(61)
    w = lambda *shape, s=0.02: (s * torch.randn(*shape, device="cuda", generator=g)).bfloat16()
    n = 3 * heads * 128
    w_t, w_i, b_t, b_i = w(n, hidden), w(n, hidden), w(n, s=0.5), w(n, s=0.5)
    nq_t, nk_t, nq_i, nk_i = ((1 + w(128, s=0.1)).contiguous() for _ in range(4))
    hl = heads // world
    outs = []
    for grouped in (False, True):
        recv = [[torch.full((world * ls, hl, 128), float("nan"), device="cuda", dtype=torch.bfloat16)
                 for _ in range(world)] for _ in range(3)]
        ptrs = [[recv[t][r].data_ptr() for r in range(world)] for t in range(3)]
        gx = torch.Generator(device="cuda").manual_seed(62)
        for r in range(world):
            x_t = torch.randn(t_loc, hidden, device="cuda", generator=gx).bfloat16()
            x_i = torch.randn(i_loc, hidden, device="cuda", generator=gx).bfloat16()
            rows = torch.arange(r * ls, (r + 1) * ls, device="cuda")
            table = rope_table(torch.stack((rows // 100, (rows // 10) % 10, rows % 10), dim=1), [16, 56, 56])
            common = dict(world=world, rank=r, seq_local=ls, seg0=t_loc, norm_mode=_lib.NORM_HEAD, eps=eps,
                          rope=table)
            streams = [dict(x=x_t, w_qkv=w_t, bias=b_t, norm_q_w=nq_t, norm_k_w=nk_t, row0=0),
                       dict(x=x_i, w_qkv=w_i, bias=b_i, norm_q_w=nq_i, norm_k_w=nk_i, row0=t_loc)]
            if grouped:
                qkv_gemm_prologue_scatter_streams(streams, ptrs, **common)
            else:
                for st in streams:
                    if st["x"].shape[0]:
                        qkv_gemm_prologue_scatter(st["x"], st["w_qkv"], ptrs, row0=st["row0"], bias=st["bias"],
                                                  norm_q_w=st["norm_q_w"], norm_k_w=st["norm_k_w"], **common)
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        outs.append(recv)
    for t in range(3):
        for r in range(world):
            assert not torch.isnan(outs[1][t][r].float()).any(), f"tensor {t} rank {r}: rows left unwritten"
            assert torch.equal(outs[0][t][r], outs[1][t][r]), f"tensor {t} rank {r}"
