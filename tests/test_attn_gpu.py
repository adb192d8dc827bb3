"""Parity of the tcgen05 attention kernel against an fp32 torch reference.

Tolerances are the ones the path is held to: bf16 output max-abs <= 2e-2 and
rel-L2 <= 5e-3 against fp32 softmax(QK^T/sqrt(D))V; FP8-e4m3 rel-L2 <= 3e-2;
LSE (natural log, fp32) within 2e-3 absolute.
"""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

BF16_MAX_ABS = 2e-2
BF16_REL_L2 = 5e-3
FP8_REL_L2 = 3e-2
LSE_ABS = 2e-3


def reference_attention(q, k, v, scale=None, chunk=2048):
    """fp32 softmax(scale * q k^T) v and natural-log LSE, (B,L,H,D) layout."""
    b, lq, h, d = q.shape
    hkv = k.shape[2]
    scale = scale or 1.0 / math.sqrt(d)
    rep = h // hkv
    kf = k.float().repeat_interleave(rep, dim=2).permute(0, 2, 3, 1)  # B H D Lk
    vf = v.float().repeat_interleave(rep, dim=2).permute(0, 2, 1, 3)  # B H Lk D
    outs, lses = [], []
    for s in range(0, lq, chunk):
        qc = q[:, s:s + chunk].float().permute(0, 2, 1, 3)  # B H c D
        logits = torch.matmul(qc, kf) * scale
        lse = torch.logsumexp(logits, dim=-1)
        p = torch.softmax(logits, dim=-1)
        outs.append(torch.matmul(p, vf).permute(0, 2, 1, 3))
        lses.append(lse)
    return torch.cat(outs, dim=1), torch.cat(lses, dim=2)


def rel_l2(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


SHAPES = [
    # (batch, q_len, kv_len, q_heads, kv_heads)
    (1, 256, 256, 1, 1),
    (1, 128, 128, 2, 2),
    (2, 300, 77, 3, 1),
    (1, 1000, 1000, 4, 4),
    (1, 513, 2049, 2, 2),
    (1, 4096, 4096, 2, 2),
]


@pytest.mark.parametrize("shape", SHAPES)
def test_bf16_matches_fp32_reference(lib, shape):
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


def test_fast_and_safe_mma_orders_agree_bitwise(lib):
    """The fast issue order reuses S tensor memory right behind the P.V that
    reads P from it; the safe order drains first.  Same math, same bits."""
    from dgx_monarch_b200.ops import attention_fwd

    g = torch.Generator(device="cuda").manual_seed(1)
    q, k, v = (torch.randn(1, 2048, 4, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    fast, fast_lse = attention_fwd(q, k, v)
    safe, safe_lse = attention_fwd(q, k, v, safe_order=True)
    torch.cuda.synchronize()
    assert torch.equal(fast, safe)
    assert torch.equal(fast_lse, safe_lse)


def test_fp32_output_and_strided_inputs(lib):
    from dgx_monarch_b200.ops import attention_fwd

    g = torch.Generator(device="cuda").manual_seed(2)
    # q/k/v as views into one packed (B, L, 3, H, D) projection output.
    qkv = torch.randn(1, 700, 3, 4, 128, device="cuda", generator=g).bfloat16()
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    out, lse = attention_fwd(q, k, v, out_dtype=torch.float32, softmax_scale=0.05)
    torch.cuda.synchronize()
    ref, ref_lse = reference_attention(q, k, v, scale=0.05)
    assert out.dtype == torch.float32
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS


def quantize_e4m3_per_head(x):
    """Per-head fp32 absmax scale (amax/448) and e4m3 values, (B,L,H,D)."""
    amax = x.float().abs().amax(dim=(0, 1, 3)).clamp_min(1e-12)
    scale = (amax / 448.0).contiguous()
    q8 = (x.float() / scale.view(1, 1, -1, 1)).to(torch.float8_e4m3fn)
    return q8, scale


def fp8_references(q, k, v):
    """(SDPA over the per-head e4m3 rounding of q, k, v; the rel-L2 of that
    against SDPA over q, k, v themselves): the reference an e4m3 kernel is held
    to, and the floor its input format alone sets against the activations."""
    deq = [x.float() * s.view(1, 1, -1, 1) for x, s in (quantize_e4m3_per_head(t) for t in (q, k, v))]
    ref_deq, _ = reference_attention(*deq)
    ref_act, _ = reference_attention(q, k, v)
    return ref_deq, rel_l2(ref_deq, ref_act)


@pytest.mark.parametrize("shape", [(1, 256, 256, 2, 2), (2, 4608, 4608, 3, 3), (1, 1000, 333, 4, 2)])
def test_fp8_matches_sdpa_within_3e2(lib, shape):
    from dgx_monarch_b200.ops import attention_fwd

    b, lq, lk, h, hkv = shape
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(b, lq, h, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).bfloat16()
    q8, qs = quantize_e4m3_per_head(q)
    k8, ks = quantize_e4m3_per_head(k)
    v8, vs = quantize_e4m3_per_head(v)
    out, lse = attention_fwd(q8, k8, v8, q_descale=qs, k_descale=ks, v_descale=vs)
    torch.cuda.synchronize()
    # The contract: SDPA over the same e4m3 inputs (dequantized with their
    # per-head scales) -- the kernel's own error, P quantization included.
    deq = [x.float() * s.view(1, 1, -1, 1) for x, s in ((q8, qs), (k8, ks), (v8, vs))]
    ref, ref_lse = reference_attention(*deq)
    assert out.dtype == torch.bfloat16
    assert rel_l2(out, ref) <= FP8_REL_L2
    assert (lse - ref_lse).abs().max().item() <= 5 * LSE_ABS
    # Against the unquantized bf16 activations the three e4m3 roundings alone
    # set a floor (about 4-5 % for N(0,1) data); the kernel adds at most its own 3e-2.
    ref_bf16, _ = reference_attention(q, k, v)
    floor = rel_l2(ref, ref_bf16)
    assert rel_l2(out, ref_bf16) <= floor + FP8_REL_L2


def test_lse_merge_reconstructs_full_attention(lib):
    """Attention over four key blocks, merged, equals attention over all keys."""
    from dgx_monarch_b200.ops import attention_fwd, lse_merge

    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(1, 1000, 3, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(1, 4 * 384, 3, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(1, 4 * 384, 3, 128, device="cuda", generator=g).bfloat16()
    parts = [attention_fwd(q, k[:, i * 384:(i + 1) * 384].contiguous(),
                           v[:, i * 384:(i + 1) * 384].contiguous(), out_dtype=torch.float32)
             for i in range(4)]
    out, lse = lse_merge([p[0] for p in parts], [p[1] for p in parts])
    torch.cuda.synchronize()
    ref, ref_lse = reference_attention(q, k, v)
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS


def test_invalid_arguments_raise_before_launch(lib):
    from dgx_monarch_b200._lib import DgxmError
    from dgx_monarch_b200.ops import attention_fwd

    q = torch.randn(1, 64, 2, 96, device="cuda").bfloat16()
    with pytest.raises(DgxmError, match="head_dim"):
        attention_fwd(q, q, q)
    q = torch.randn(1, 64, 3, 128, device="cuda").bfloat16()
    k = torch.randn(1, 64, 2, 128, device="cuda").bfloat16()
    with pytest.raises(DgxmError, match="divisible"):
        attention_fwd(q, k, k)


def test_keep_masks_exclude_pad_rows_exactly(lib):
    """In-kernel pad exclusion: attention over the kept rows only, zeros (and
    LSE -inf) at dropped query rows -- adapters/usp_pad_exclusion.py:112-137."""
    from dgx_monarch_b200.ops import attention_fwd_ext, keep_bits

    g = torch.Generator(device="cuda").manual_seed(31)
    rows = 700
    q, k, v = (torch.randn(1, rows, 3, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    drop = [0, 5, 127, 128, 255, 256, 311, 699]
    kk = keep_bits(rows, drop, q.device)
    out, lse = attention_fwd_ext(q, k, v, key_keep=kk, query_keep=kk,
                                 lse=torch.empty(1, 3, rows, device="cuda"))
    torch.cuda.synchronize()
    keep = [i for i in range(rows) if i not in drop]
    ref, ref_lse = reference_attention(q[:, keep], k[:, keep], v[:, keep])
    assert (out[:, keep].float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(out[:, keep], ref) <= BF16_REL_L2
    assert torch.equal(out[:, drop], torch.zeros_like(out[:, drop]))
    assert (lse[:, :, keep] - ref_lse).abs().max().item() <= LSE_ABS
    assert torch.isinf(lse[:, :, drop]).all()


def test_key_mask_over_whole_blocks_and_cross_attention(lib):
    """Keys dropped over entire 128-key blocks, and a key side that pads
    while the query side does not."""
    from dgx_monarch_b200.ops import attention_fwd_ext, keep_bits

    g = torch.Generator(device="cuda").manual_seed(37)
    q = torch.randn(1, 300, 2, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(1, 600, 2, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(1, 600, 2, 128, device="cuda", generator=g).bfloat16()
    drop = list(range(0, 256)) + [599]
    out, _ = attention_fwd_ext(q, k, v, key_keep=keep_bits(600, drop, q.device))
    torch.cuda.synchronize()
    keep = [i for i in range(600) if i not in drop]
    ref, _ = reference_attention(q, k[:, keep], v[:, keep])
    assert rel_l2(out, ref) <= BF16_REL_L2


def test_query_group_bias_matches_sdpa_with_additive_mask(lib):
    """adapters/usp_query_bias.py:109-130: each query group attends the full
    keys under its own additive bias (zero-extended past its keys): a key row
    shared over heads, no bias, a per-head key row with -inf keys, and a
    per-query-row bias (the LTX tracked-guide rectangle)."""
    from dgx_monarch_b200.ops import attention_fwd_ext

    g = torch.Generator(device="cuda").manual_seed(41)
    rows, heads = 650, 2
    q, k, v = (torch.randn(1, rows, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    b0 = torch.randn(1, 1, 1, 300, device="cuda", generator=g) * 2.0     # shared over heads, 300 keys
    b2 = torch.randn(1, heads, 1, rows, device="cuda", generator=g)       # per head, all keys
    b2[..., 10:20] = float("-inf")
    b3 = torch.zeros(1, 1, 130, rows, device="cuda")                      # one weight per query row
    b3[..., :400] = torch.log(torch.rand(1, 1, 130, 1, device="cuda", generator=g) + 0.05)
    groups = [(0, 100, b0), (100, 260, None), (260, 520, b2), (520, rows, b3)]
    out, _ = attention_fwd_ext(q, k, v, bias_groups=groups)
    torch.cuda.synchronize()
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    for start, end, bias in groups:
        logits = qf[:, :, start:end] @ kf.transpose(-1, -2) / math.sqrt(128)
        if bias is not None:
            full = torch.zeros(1, bias.shape[1], bias.shape[2], rows, device="cuda")
            full[..., :bias.shape[3]] = bias
            logits = logits + full
        ref = (torch.softmax(logits, -1) @ vf).transpose(1, 2)
        assert rel_l2(out[:, start:end], ref) <= BF16_REL_L2


def test_fp8_extras_bias_groups_and_keep_masks(lib):
    """The e4m3 extras kernel: a bias is in logit units, so it is added to
    the raw e4m3 products divided by the softmax scale and the q and k
    descales; key pads drop out and query pads come back as zeros.  Held to
    fp32 attention over the dequantized inputs with the same biases."""
    from dgx_monarch_b200.ops import attention_fwd_ext, keep_bits

    g = torch.Generator(device="cuda").manual_seed(43)
    rows, heads = 520, 2
    q, k, v = (torch.randn(1, rows, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    (q8, qs), (k8, ks), (v8, vs) = (quantize_e4m3_per_head(t) for t in (q, k, v))
    b0 = torch.randn(1, 1, 1, 300, device="cuda", generator=g) * 2.0
    b2 = torch.randn(1, heads, 1, rows, device="cuda", generator=g)
    groups = [(0, 200, b0), (200, 300, None), (300, rows, b2)]
    drop = [5, 77, 519]
    keep = keep_bits(rows, drop, q.device)
    out, _ = attention_fwd_ext(q8, k8, v8, bias_groups=groups, key_keep=keep, query_keep=keep,
                               q_descale=qs, k_descale=ks, v_descale=vs)
    torch.cuda.synchronize()
    deq = [x.float() * sc.view(1, 1, -1, 1) for x, sc in ((q8, qs), (k8, ks), (v8, vs))]
    qf, kf, vf = (t.transpose(1, 2) for t in deq)
    live = torch.ones(rows, dtype=torch.bool, device="cuda")
    live[drop] = False
    for start, end, bias in groups:
        logits = qf[:, :, start:end] @ kf.transpose(-1, -2) / math.sqrt(128)
        if bias is not None:
            full = torch.zeros(1, bias.shape[1], bias.shape[2], rows, device="cuda")
            full[..., :bias.shape[3]] = bias
            logits = logits + full
        logits[..., ~live] = float("-inf")
        ref = (torch.softmax(logits, -1) @ vf).transpose(1, 2)
        ref[:, ~live[start:end]] = 0
        assert rel_l2(out[:, start:end], ref) <= FP8_REL_L2
    assert torch.count_nonzero(out[:, drop]).item() == 0


def test_row_with_only_excluded_keys_in_leading_blocks(lib):
    """One query row whose first 384 keys are excluded by its bias, beside
    rows that see every key: the row must attend the remaining keys (its
    running maximum stays -inf while the warp's other rows rescale)."""
    from dgx_monarch_b200.ops import attention_fwd_ext

    g = torch.Generator(device="cuda").manual_seed(43)
    rows = 600
    q, k, v = (torch.randn(1, rows, 2, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    rect = torch.zeros(1, 1, 64, rows, device="cuda")
    rect[:, :, 5, :384] = torch.finfo(torch.float32).min
    rect[:, :, 40, :] = float("-inf")  # a row that sees no key at all: zeros, as an empty softmax
    out, _ = attention_fwd_ext(q, k, v, bias_groups=[(0, 64, rect)])
    torch.cuda.synchronize()
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    logits = qf[:, :, :64] @ kf.transpose(-1, -2) / math.sqrt(128) + rect.clamp_min(-1e30)
    ref = (torch.softmax(logits, -1) @ vf).transpose(1, 2)
    keep = [i for i in range(64) if i != 40]
    assert rel_l2(out[:, keep], ref[:, keep]) <= BF16_REL_L2
    assert (out[:, 5].float() - ref[:, 5]).abs().max().item() <= BF16_MAX_ABS
    assert torch.equal(out[:, 40], torch.zeros_like(out[:, 40]))
    rest, _ = reference_attention(q[:, 64:], k, v)
    assert rel_l2(out[:, 64:], rest) <= BF16_REL_L2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_cfg_combine_is_bit_exact_against_torch(lib, dtype):
    """uncond + (cond - uncond) * cfg (comfy's default cfg_function, as the
    dual-model CFG split runs it) against torch's unfused expression, with a
    tail that does not fill a 16-byte vector and an output aliasing cond."""
    from dgx_monarch_b200.cfg import cfg_combine

    g = torch.Generator(device="cuda").manual_seed(47)
    for n in (16 * 128 * 128, 1003):
        c = torch.randn(n, device="cuda", generator=g).to(dtype)
        u = torch.randn(n, device="cuda", generator=g).to(dtype)
        want = u + (c - u) * 5.5
        assert torch.equal(cfg_combine(c, u, 5.5), want)
        assert torch.equal(cfg_combine(c, u, 5.5, out=c), want)


@pytest.mark.parametrize("heads,kv_heads,groups", [(8, 8, 4), (8, 4, 2), (6, 6, 3)])
def test_host_streamed_attention_equals_one_device_call(lib, heads, kv_heads, groups):
    """Pinned host tensors streamed through the device by head groups give the
    same bits as one attention call over the whole device tensors."""
    from dgx_monarch_b200.ops import HostStreamedAttention, attention_fwd

    g = torch.Generator(device="cuda").manual_seed(57)
    q = torch.randn(2, 1000, heads, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(2, 1300, kv_heads, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(2, 1300, kv_heads, 128, device="cuda", generator=g).bfloat16()
    want, _ = attention_fwd(q, k, v, return_lse=False)
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.full(q.shape, float("nan"), dtype=torch.bfloat16).pin_memory()
    streamed = HostStreamedAttention(2, 1000, 1300, heads, kv_heads, device=q.device, groups=groups)
    for _ in range(2):  # a second call reuses the device buffers and streams
        streamed(hq, hk, hv, hout)
        torch.cuda.synchronize()
        assert torch.equal(hout.cuda(), want)


def test_buffers_that_do_not_cover_the_launch_are_refused(lib):
    """A caller-given output, LSE or descale that the kernel would overrun, or a
    host tensor, is refused before anything launches."""
    from dgx_monarch_b200.cfg import cfg_combine
    from dgx_monarch_b200.ops import attention_fwd, attention_fwd_ext
    from dgx_monarch_b200.prologue import quantize_e4m3_per_head

    q, k, v = (torch.randn(1, 64, 2, 128, device="cuda").bfloat16() for _ in range(3))
    bf16 = {"device": "cuda", "dtype": torch.bfloat16}
    with pytest.raises(ValueError, match="out"):
        attention_fwd(q, k, v, out=torch.empty(1, 32, 2, 128, **bf16))
    with pytest.raises(ValueError, match="lse"):
        attention_fwd(q, k, v, lse=torch.empty(1, 2, 32, device="cuda"))
    with pytest.raises(ValueError, match="lse"):
        attention_fwd_ext(q, k, v, lse=torch.empty(1, 64, 2, device="cuda"))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        attention_fwd(q, k, v, out=torch.empty(1, 64, 2, 128, dtype=torch.bfloat16))
    q8 = torch.empty(1, 64, 2, 128, device="cuda", dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="k_descale"):
        attention_fwd(q8, q8, q8, q_descale=torch.ones(2, device="cuda"), k_descale=torch.ones(1, device="cuda"),
                      v_descale=torch.ones(2, device="cuda"))
    with pytest.raises(ValueError, match="out"):
        quantize_e4m3_per_head(q, out=q8[:, :32])
    with pytest.raises(ValueError, match="descale"):
        quantize_e4m3_per_head(q, descale=torch.empty(1, device="cuda"))
    c = torch.randn(1000, device="cuda")
    with pytest.raises(ValueError, match="out"):
        cfg_combine(c, c, 3.0, out=torch.empty(500, device="cuda"))
    torch.cuda.synchronize()


def test_empty_inputs_return_without_a_launch(lib):
    """No query rows or an empty batch give empty results; an empty key axis
    has no defined output and is refused; an empty merge and an empty
    scatter do nothing.  None of these reaches a kernel."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ops import attention_fwd, lse_merge
    from dgx_monarch_b200.ulysses import ulysses_scatter

    bf16 = {"device": "cuda", "dtype": torch.bfloat16}
    k = torch.randn(1, 64, 2, 128, device="cuda").bfloat16()
    out, lse = attention_fwd(torch.empty(1, 0, 2, 128, **bf16), k, k)
    assert out.shape == (1, 0, 2, 128) and lse.shape == (1, 2, 0)
    none = torch.empty(0, 16, 2, 128, **bf16)
    out, _ = attention_fwd(none, none, none)
    assert out.shape == (0, 16, 2, 128)
    no_keys = torch.empty(1, 0, 2, 128, **bf16)
    with pytest.raises(_lib.DgxmError, match="empty key axis"):
        attention_fwd(torch.randn(1, 16, 2, 128, device="cuda").bfloat16(), no_keys, no_keys)
    parts = [torch.empty(1, 0, 2, 128, device="cuda") for _ in range(2)]
    lses = [torch.empty(1, 2, 0, device="cuda") for _ in range(2)]
    merged, merged_lse = lse_merge(parts, lses)
    assert merged.shape == (1, 0, 2, 128) and merged_lse.shape == (1, 2, 0)
    recv = torch.zeros(1, 8, 2, 128, **bf16)
    ulysses_scatter([torch.empty(1, 0, 4, 128, **bf16)] * 3, [[recv.data_ptr()] * 2] * 3, world=2, rank=0)
    torch.cuda.synchronize()
    assert recv.abs().max().item() == 0.0
    assert _lib.device_error() == 0


# fp16 runs the 16-bit path in its own format (Q, K, V and P in fp16, fp16 or
# fp32 output): fp16's 10 mantissa bits hold it well inside the bf16 bounds.
F16_MAX_ABS = 1e-2
F16_REL_L2 = 2e-3


@pytest.mark.parametrize("shape", [(1, 1000, 1000, 4, 4), (2, 300, 77, 3, 1), (1, 513, 2049, 2, 2)])
def test_fp16_runs_natively_and_matches_fp32_reference(lib, shape):
    """The reference's flash path takes fp16 models' q/k/v as they are
    (adapters/wan_ring_full_context.py:10); so does this kernel."""
    from dgx_monarch_b200.ops import attention_fwd

    b, lq, lk, h, hkv = shape
    g = torch.Generator(device="cuda").manual_seed(16)
    q = torch.randn(b, lq, h, 128, device="cuda", generator=g).half()
    k = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).half()
    v = torch.randn(b, lk, hkv, 128, device="cuda", generator=g).half()
    out, lse = attention_fwd(q, k, v)
    out32, lse32 = attention_fwd(q, k, v, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16 and out32.dtype == torch.float32
    ref, ref_lse = reference_attention(q, k, v)
    for got in (out, out32):
        assert (got.float() - ref).abs().max().item() <= F16_MAX_ABS
        assert rel_l2(got, ref) <= F16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS
    assert (lse - lse32).abs().max().item() <= 1e-5
    # Computing in fp16 is closer to the fp16 inputs' exact attention than
    # rounding them to bf16 first would be.
    via_bf16, _ = attention_fwd(q.bfloat16(), k.bfloat16(), v.bfloat16())
    assert rel_l2(out, ref) < rel_l2(via_bf16, ref)


def test_fp16_extras_and_merge(lib):
    """fp16 through the extras kernel (pad keep bits) and the LSE merge of
    fp16 and fp32 parts."""
    from dgx_monarch_b200.ops import attention_fwd, attention_fwd_ext, keep_bits, lse_merge

    g = torch.Generator(device="cuda").manual_seed(17)
    rows = 700
    q, k, v = (torch.randn(1, rows, 3, 128, device="cuda", generator=g).half() for _ in range(3))
    drop = [0, 127, 128, 699]
    kk = keep_bits(rows, drop, q.device)
    out, _ = attention_fwd_ext(q, k, v, key_keep=kk, query_keep=kk)
    torch.cuda.synchronize()
    keep = [i for i in range(rows) if i not in drop]
    ref, _ = reference_attention(q[:, keep], k[:, keep], v[:, keep])
    assert out.dtype == torch.float16
    assert rel_l2(out[:, keep], ref) <= F16_REL_L2
    assert torch.equal(out[:, drop], torch.zeros_like(out[:, drop]))
    full_ref, full_lse = reference_attention(q, k, v)
    for part_dtype in (torch.float16, torch.float32):
        parts = [attention_fwd(q, k[:, i * 350:(i + 1) * 350].contiguous(), v[:, i * 350:(i + 1) * 350].contiguous(),
                               out_dtype=part_dtype) for i in range(2)]
        merged, lse = lse_merge([p[0] for p in parts], [p[1] for p in parts], out_dtype=torch.float16)
        torch.cuda.synchronize()
        assert merged.dtype == torch.float16
        assert rel_l2(merged, full_ref) <= F16_REL_L2
        assert (lse - full_lse).abs().max().item() <= LSE_ABS


def test_mixed_16bit_formats_are_refused(lib):
    from dgx_monarch_b200._lib import DgxmError
    from dgx_monarch_b200.ops import attention_fwd, lse_merge

    q = torch.randn(1, 64, 2, 128, device="cuda").half()
    with pytest.raises(DgxmError, match="output dtype"):
        attention_fwd(q, q, q, out_dtype=torch.bfloat16)
    parts = [torch.zeros(1, 64, 2, 128, device="cuda", dtype=torch.float16)]
    with pytest.raises(DgxmError, match="f16 parts into a bf16"):
        lse_merge(parts, [torch.zeros(1, 2, 64, device="cuda")], out_dtype=torch.bfloat16)


@pytest.mark.parametrize("dtype,shape,out_f32", [
    (torch.bfloat16, (1, 256, 256, 2, 2), False),
    (torch.bfloat16, (2, 1000, 777, 4, 2), True),     # ragged tiles, GQA, fp32 out
    (torch.float16, (1, 4096, 4096, 3, 3), False),
    (torch.bfloat16, (1, 9000, 9000, 2, 1), False),   # 71 key blocks, MQA
])
def test_head_dim_64_matches_fp32_reference(lib, dtype, shape, out_f32):
    """The head-dim-64 kernel (16-bit inputs): Q·Kᵀ over 64 dims, O of 64
    columns, 8 K/V stages of 16 KB; against fp32 attention, out and LSE."""
    from dgx_monarch_b200.ops import attention_fwd

    b, lq, lk, h, hkv = shape
    g = torch.Generator(device="cuda").manual_seed(lq + 64)
    q = torch.randn(b, lq, h, 64, device="cuda", generator=g).to(dtype)
    k = torch.randn(b, lk, hkv, 64, device="cuda", generator=g).to(dtype)
    v = torch.randn(b, lk, hkv, 64, device="cuda", generator=g).to(dtype)
    out, lse = attention_fwd(q, k, v, out_dtype=torch.float32 if out_f32 else None)
    torch.cuda.synchronize()
    ref, ref_lse = reference_attention(q, k, v)
    tol = BF16_REL_L2 if dtype == torch.bfloat16 else 2e-3
    assert out.shape == (b, lq, h, 64)
    assert out.dtype == (torch.float32 if out_f32 else dtype)
    assert rel_l2(out, ref) <= tol
    assert (out.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS


def test_head_dim_64_extras_and_padding_agree(lib):
    """Keep masks and a bias group on the head-dim-64 kernel, and the same
    heads zero-padded to 128 on the 128 kernel: both against fp32 attention."""
    from dgx_monarch_b200.ops import attention_fwd, attention_fwd_ext, keep_bits

    g = torch.Generator(device="cuda").manual_seed(640)
    rows, heads = 700, 2
    q, k, v = (torch.randn(1, rows, heads, 64, device="cuda", generator=g).bfloat16() for _ in range(3))
    bias = torch.randn(1, heads, 1, rows, device="cuda", generator=g)
    drop = [3, 350, 699]
    keep = keep_bits(rows, drop, q.device)
    out, _ = attention_fwd_ext(q, k, v, key_keep=keep, query_keep=keep, bias_groups=[(100, 400, bias)])
    torch.cuda.synchronize()
    live = torch.ones(rows, dtype=torch.bool, device="cuda")
    live[drop] = False
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    logits = qf @ kf.transpose(-1, -2) / math.sqrt(64)
    logits[:, :, 100:400] += bias
    logits[..., ~live] = float("-inf")
    ref = (torch.softmax(logits, -1) @ vf).transpose(1, 2)
    ref[:, ~live] = 0
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert torch.count_nonzero(out[:, drop]).item() == 0
    pad = [torch.nn.functional.pad(t, (0, 64)) for t in (q, k, v)]
    padded, _ = attention_fwd(*pad, softmax_scale=1.0 / math.sqrt(64))
    native, _ = attention_fwd(q, k, v)
    torch.cuda.synchronize()
    assert rel_l2(native, padded[..., :64]) <= BF16_REL_L2
