"""The collective kernels on one GPU, against the oracle.

The store halves of the gathers run with the ranks emulated: every emulated
rank's destination buffers live on the one device and each source rank's
stores are their own launch, so no kernel waits on another.  The collectives
whose barrier or exchange runs inside the same kernel (the shared NVFP4
scale, the CFG prediction gather) run on a world-1 peer window.  Layouts are
bit-exact against the oracle's restatements of the reference's collectives:
sp_gather (adapters/base.py:126-131), the full-context K/V gather
(adapters/wan_ring_full_context.py:203-295), the ring's block order
(the xfuser ring reached from adapters/base.py:320), the shared activation
scale (adapters/quant_activation_scale.py:222-246) and the CFG all-gather
(adapters/cfg_parallel.py:293-301).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import usp
from tests.test_attn_gpu import BF16_REL_L2, rel_l2

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous()
    return t.view(torch.int16 if t.element_size() == 2 else torch.int32).cpu().numpy()


@pytest.mark.parametrize("world,batch,seq_local,orig_len,row,dtype", [
    (2, 1, 40, 80, 3072, torch.bfloat16),     # no pad
    (4, 2, 13, 49, 3072, torch.bfloat16),     # the last rank's 3 pad rows are trimmed
    (8, 1, 1216, 9728, 3072, torch.bfloat16), # the Flux/Krea2 token stream at Ulysses-8
    (3, 2, 7, 19, 40, torch.float32),         # 160-byte rows
    (8, 1, 5, 33, 8, torch.float16),          # 16-byte rows, most ranks all pad
])
def test_seq_gather_stores_are_the_trimmed_all_gather(lib, world, batch, seq_local, orig_len, row, dtype):
    from dgx_monarch_b200.shard import seq_gather_store

    g = torch.Generator(device="cuda").manual_seed(world * 100 + seq_local)
    chunks = [torch.randn(batch, seq_local, row, device="cuda", generator=g).to(dtype) for _ in range(world)]
    dst = [torch.full((batch, orig_len, row), float("nan"), device="cuda", dtype=dtype) for _ in range(world)]
    for r in range(world):
        seq_gather_store(chunks[r], orig_len, [d.data_ptr() for d in dst], world=world, rank=r)
    torch.cuda.synchronize()
    want = usp.sp_gather([_bits(c) for c in chunks], orig_len)
    for r in range(world):
        assert np.array_equal(_bits(dst[r]), want)


@pytest.mark.parametrize("world,batch,rows,heads,dtype,strided", [
    (2, 1, 300, 4, torch.bfloat16, False),
    (4, 2, 77, 2, torch.float16, True),
    (8, 1, 129, 5, torch.bfloat16, True),
])
def test_kv_gather_stores_rank_major_slots(lib, world, batch, rows, heads, dtype, strided):
    from dgx_monarch_b200.ring import kv_gather_store

    g = torch.Generator(device="cuda").manual_seed(rows)
    blocks = []
    for _ in range(world):
        if strided:  # k and v as views of one packed (B, L, 2, H, D) projection output
            kv = torch.randn(batch, rows, 2, heads, 128, device="cuda", generator=g).to(dtype)
            blocks.append((kv[:, :, 0], kv[:, :, 1]))
        else:
            blocks.append(tuple(torch.randn(batch, rows, heads, 128, device="cuda", generator=g).to(dtype)
                                for _ in range(2)))
    full = [[torch.full((batch, world * rows, heads, 128), float("nan"), device="cuda", dtype=dtype)
             for _ in range(world)] for _ in range(2)]
    for r in range(world):
        kv_gather_store(blocks[r][0], blocks[r][1], [f.data_ptr() for f in full[0]],
                        [f.data_ptr() for f in full[1]], world=world, rank=r)
    torch.cuda.synchronize()
    for t in range(2):
        want = usp.full_context_gather([_bits(b[t]) for b in blocks])
        for r in range(world):
            assert np.array_equal(_bits(full[t][r]), want)


def test_emulated_ring_follows_the_oracle_block_order(lib):
    """Four ranks' ring steps on one GPU, each rank attending the block of
    rank (r - t) mod R at step t (fp32 partials, LSE merge), against the
    oracle's float64 ring attention."""
    from dgx_monarch_b200.ops import attention_fwd, lse_merge

    world, rows, heads = 4, 200, 2
    g = torch.Generator(device="cuda").manual_seed(4)
    q, k, v = ([torch.randn(1, rows, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(world)]
               for _ in range(3))
    f64 = lambda ts: [t.double().cpu().numpy() for t in ts]
    want = usp.ring_attention(f64(q), f64(k), f64(v))
    for r in range(world):
        parts = [attention_fwd(q[r], k[(r - t) % world], v[(r - t) % world], out_dtype=torch.float32)
                 for t in range(world)]
        out, lse = lse_merge([p[0] for p in parts], [p[1] for p in parts])
        torch.cuda.synchronize()
        assert rel_l2(out, torch.from_numpy(want[r][0]).cuda()) <= BF16_REL_L2
        assert np.abs(lse.double().cpu().numpy() - want[r][1]).max() <= 2e-3


def test_emulated_fp8_ring_with_per_block_scales(lib):
    """The e4m3 ring's arithmetic on one GPU: every block quantised over its
    own rows, each step an e4m3 attention with fp32 partials under the
    block's descales, then the LSE merge; against fp32 attention over the
    per-block dequantized axis."""
    from dgx_monarch_b200.ops import attention_fwd, lse_merge
    from tests.test_attn_gpu import FP8_REL_L2, quantize_e4m3_per_head, reference_attention

    world, rows, heads = 3, 300, 2
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = ([torch.randn(1, rows, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(world)]
               for _ in range(3))
    q8, k8, v8 = ([quantize_e4m3_per_head(t) for t in ts] for ts in (q, k, v))
    deq = lambda qs: torch.cat([x.float() * sc.view(1, 1, -1, 1) for x, sc in qs], dim=1)
    kd, vd = deq(k8), deq(v8)
    for r in range(world):
        parts = [attention_fwd(q8[r][0], k8[(r - t) % world][0], v8[(r - t) % world][0], q_descale=q8[r][1],
                               k_descale=k8[(r - t) % world][1], v_descale=v8[(r - t) % world][1],
                               out_dtype=torch.float32) for t in range(world)]
        out, lse = lse_merge([p[0] for p in parts], [p[1] for p in parts])
        torch.cuda.synchronize()
        ref, ref_lse = reference_attention(deq([q8[r]]), kd, vd)
        assert rel_l2(out, ref) <= FP8_REL_L2
        assert (lse - ref_lse).abs().max().item() <= 5e-3


def test_fp8_ring_entry_at_world_one_and_its_refusals(lib):
    """A one-rank e4m3 ring is one e4m3 attention (bit-identical); e4m3
    inputs without descales, descales with 16-bit inputs, and 16-bit inputs
    through the e4m3 entry are refused before any launch."""
    import ctypes

    from dgx_monarch_b200 import _lib as L
    from dgx_monarch_b200.ops import attention_fwd, attn_desc
    from dgx_monarch_b200.ring import RingAttention
    from tests.test_attn_gpu import quantize_e4m3_per_head

    g = torch.Generator(device="cuda").manual_seed(6)
    q, k, v = (torch.randn(1, 256, 2, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    (q8, qs), (k8, ks), (v8, vs) = (quantize_e4m3_per_head(t) for t in (q, k, v))
    ring = RingAttention(world=1, rank=0, batch=1, q_len=256, kv_len=256, heads=2, kv_heads=2, head_dim=128,
                         device=q.device, generation=32, dtype=torch.float8_e4m3fn)
    try:
        out, _ = ring.forward(q8, k8, v8, q_descale=qs, k_descale=ks, v_descale=vs)
        want, _ = attention_fwd(q8, k8, v8, q_descale=qs, k_descale=ks, v_descale=vs)
        torch.cuda.synchronize()
        assert out.dtype == torch.bfloat16 and torch.equal(out, want)
        lib_ = L.load()
        stream = torch.cuda.current_stream().cuda_stream
        o = torch.empty_like(q)
        d8 = attn_desc(q8, k8, v8, o, None)
        rc = lib_.dgxm_ring_attn_fwd(ring.windows._handle, ctypes.byref(d8), q8.data_ptr(), k8.data_ptr(),
                                     v8.data_ptr(), o.data_ptr(), None, ring.workspace.data_ptr(),
                                     ring.workspace_bytes, stream)
        assert rc == L.DGXM_ERR_INVALID and b"descales" in lib_.dgxm_last_error_message()
        d16 = attn_desc(q, k, v, o, None)
        rc = lib_.dgxm_ring_attn_fwd_fp8(ring.windows._handle, ctypes.byref(d16), q.data_ptr(), k.data_ptr(),
                                         v.data_ptr(), qs.data_ptr(), ks.data_ptr(), vs.data_ptr(), o.data_ptr(),
                                         None, ring.workspace.data_ptr(), ring.workspace_bytes, stream)
        assert rc == L.DGXM_ERR_INVALID and b"e4m3" in lib_.dgxm_last_error_message()
    finally:
        ring.close()


@pytest.mark.parametrize("dtype,rows,cols,stride", [
    (torch.bfloat16, 9728, 9216, 9216),   # the Flux/Krea2 activation, 16-byte rows
    (torch.float16, 1000, 1000, 1003),    # rows that break 16-byte alignment
    (torch.float32, 3, 5, 5),
    (torch.bfloat16, 0, 64, 64),          # an empty shard
])
def test_shared_scale_kernels_on_one_rank(lib, dtype, rows, cols, stride):
    """The local amax kernel and the exchange kernel on a world-1 window: the
    scale is the oracle's over this one shard, bit for bit, and a NaN
    propagates."""
    from dgx_monarch_b200.shard import NVFP4_SCALE_DIVISOR, SharedActivationScale

    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    base = torch.randn(max(rows, 1) * stride, device="cuda", generator=g).to(dtype)
    x = base[:rows * stride].view(rows, stride)[:, :cols] if rows else torch.empty(0, cols, device="cuda", dtype=dtype)
    if rows:
        x[rows // 2, cols // 3] = 37.5
    scale = SharedActivationScale(device=x.device, generation=5)
    try:
        got = scale(x)
        torch.cuda.synchronize()
        want = usp.shared_activation_scale([x.float().cpu().numpy()], NVFP4_SCALE_DIVISOR,
                                           str(dtype).split(".")[-1])
        assert got.dtype == dtype and got.item() == want
        if rows:
            x[0, 0] = float("nan")
            assert torch.isnan(scale(x)).item()
    finally:
        scale.close()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_cfg_gather_then_combine_on_one_rank(lib, dtype):
    """The prediction gather (copy-engine stores into the window, then the
    barrier) returns the prediction bit for bit on a world-1 window, twice in
    a row (alternating buffers), and the combine over a gathered cond/uncond
    pair matches the oracle's rounding."""
    from dgx_monarch_b200.cfg import CfgGather, cfg_combine

    g = torch.Generator(device="cuda").manual_seed(9)
    pred = torch.randn(1, 16, 64, 64, device="cuda", generator=g).to(dtype)
    gather = CfgGather(pred.numel() * pred.element_size(), device=pred.device, generation=6)
    try:
        for step in range(2):
            x = pred + step
            got = gather(x)
            torch.cuda.synchronize()
            assert torch.equal(got, x)
    finally:
        gather.close()
    cond, uncond = pred, torch.randn(pred.shape, device="cuda", generator=g).to(dtype)
    got = cfg_combine(cond, uncond, 4.5)
    want = usp.cfg_combine(cond.float().cpu().numpy(), uncond.float().cpu().numpy(), 4.5,
                           str(dtype).split(".")[-1])
    assert np.array_equal(got.float().cpu().numpy(), want.astype(np.float32))


def test_store_halves_refuse_bad_destinations(lib):
    from dgx_monarch_b200._lib import DgxmError
    from dgx_monarch_b200.ring import kv_gather_store
    from dgx_monarch_b200.shard import seq_gather_store

    x = torch.zeros(1, 4, 8, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(DgxmError, match="out of range"):
        seq_gather_store(x, 8, [x.data_ptr(), x.data_ptr()], world=2, rank=2)
    with pytest.raises(DgxmError, match="not 16-byte aligned"):
        seq_gather_store(x, 8, [x.data_ptr(), x.data_ptr() + 2], world=2, rank=0)
    with pytest.raises(DgxmError, match="orig_len"):
        seq_gather_store(x, 9, [x.data_ptr(), x.data_ptr()], world=2, rank=0)
    k = torch.zeros(1, 4, 1, 128, device="cuda", dtype=torch.float32)
    with pytest.raises(DgxmError, match="bf16 or f16"):
        kv_gather_store(k, k, [k.data_ptr()], [k.data_ptr()], world=1, rank=0)


def test_ring_entry_refuses_layouts_it_cannot_merge(lib):
    """At any ring degree (here a one-rank ring) the ring entry refuses a
    strided LSE -- the merge writes (B, H, L) contiguously -- and a
    non-contiguous output, before any launch."""
    import ctypes

    from dgx_monarch_b200 import _lib as L
    from dgx_monarch_b200.ops import attn_desc
    from dgx_monarch_b200.ring import RingAttention

    q = torch.randn(1, 256, 2, 128, device="cuda").bfloat16()
    ring = RingAttention(world=1, rank=0, batch=1, q_len=256, kv_len=256, heads=2, kv_heads=2, head_dim=128,
                         device=q.device, generation=31)
    try:
        out = torch.empty_like(q)
        lse_t = torch.empty(1, 256, 2, device="cuda").transpose(1, 2)   # (B, H, L) view, strided
        desc = attn_desc(q, q, q, out, lse_t)
        stream = torch.cuda.current_stream().cuda_stream
        for entry in ("dgxm_ring_attn_fwd", "dgxm_ring_attn_fwd_noalloc"):
            fn = getattr(L.load(), entry)
            args = [ring.windows._handle, ctypes.byref(desc), q.data_ptr(), q.data_ptr(), q.data_ptr(),
                    out.data_ptr(), lse_t.data_ptr()]
            if entry == "dgxm_ring_attn_fwd":
                args += [ring.workspace.data_ptr(), ring.workspace_bytes]
            rc = fn(*args, stream)
            assert rc == L.DGXM_ERR_INVALID and b"contiguous (B, H, L) lse" in L.load().dgxm_last_error_message()
        wide = torch.empty(1, 256, 4, 128, device="cuda", dtype=torch.bfloat16)[:, :, :2]
        with pytest.raises(L.DgxmError, match="contiguous"):
            ring.forward(q, q, q, out=wide)
    finally:
        ring.close()
