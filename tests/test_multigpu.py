"""Ulysses across real GPUs: IPC peer windows, peer stores, flag barriers.

Runs only when at least two CUDA devices are visible; each rank is a child
process on its own GPU (never two ranks on one GPU, so no kernel waits on a
kernel of another launch on the same device).  NCCL carries only the window
handle exchange; NVLS stays off.
"""
from __future__ import annotations

import math
import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, q):
    """One rank.  Whatever its case does, every rank ends at the same barrier
    before reporting, so a failure on one rank never leaves another waiting
    in a collective it alone entered."""
    import torch.distributed as dist

    err = None
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from datetime import timedelta

        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=60))
        case(rank, world, dev)
    except Exception:  # pragma: no cover - reported to the parent
        err = f"rank {rank}:\n{traceback.format_exc()}"
    try:
        if dist.is_initialized():
            torch.cuda.synchronize()
            dist.barrier()
    except Exception:  # pragma: no cover
        err = (err or "") + f"rank {rank} final barrier:\n{traceback.format_exc()}"
    q.put((rank, err))
    q.close()
    q.join_thread()
    if dist.is_initialized():
        dist.destroy_process_group()


class Checks:
    """Deferred assertions: a case records failures and raises them only after
    its last collective step, so every rank takes the same steps."""

    def __init__(self, rank):
        self.rank, self.failed = rank, []

    def __call__(self, ok, what):
        if not ok:
            self.failed.append(what)

    def le(self, value, bound, what):
        """Record `what` (with the measured value) unless value <= bound."""
        value = float(value)
        if not value <= bound:
            self.failed.append(f"{what}: {value:.4g} > {bound:.4g}")

    def close(self):
        if self.failed:
            raise AssertionError(f"rank {self.rank}: " + "; ".join(self.failed))


def _spawn(case, world, limit_s=300):
    import queue
    import time

    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results, deadline = {}, time.monotonic() + limit_s
    while len(results) < world and time.monotonic() < deadline:
        try:
            rank, err = q.get(timeout=5)
            results[rank] = err
        except queue.Empty:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=60)
    for p in procs:  # only the children this call started
        if p.is_alive():
            p.terminate()
            p.join(timeout=30)
    missing = [r for r in range(world) if r not in results]
    errors = [e for e in results.values() if e]
    if missing:
        errors.append(f"ranks {missing} reported nothing (exit codes "
                      f"{[procs[r].exitcode for r in missing]})")
    assert not errors, "\n".join(errors)


def _ulysses_case(rank, world, dev):
    check = Checks(rank)
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ulysses import UlyssesAttention
    from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, reference_attention, rel_l2

    heads, ls = 4 * world, 300
    g = torch.Generator(device=dev).manual_seed(99)  # same full tensors on every rank
    q, k, v = (torch.randn(1, ls * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    mine = [x[:, rank * ls:(rank + 1) * ls].contiguous() for x in (q, k, v)]
    uly = UlyssesAttention(world=world, rank=rank, batch=1, seq_local=ls, heads=heads, head_dim=128,
                           device=dev, generation=1)
    out = None
    for _ in range(3):  # repeated steps reuse the windows and advance the barrier epoch
        out = uly.forward(*mine).clone()
    torch.cuda.synchronize()
    ref, _ = reference_attention(q, k, v)
    ref = ref[:, rank * ls:(rank + 1) * ls]
    check.le((out.float() - ref).abs().max().item(), BF16_MAX_ABS, "ulysses max abs")
    check.le(rel_l2(out, ref), BF16_REL_L2, "ulysses rel l2")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    uly.close()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_ulysses_across_gpus_matches_unsharded_attention():
    _spawn(_ulysses_case, min(torch.cuda.device_count(), 4))


def _ring_case(rank, world, dev):
    check = Checks(rank)
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ring import RingAttention
    from tests.test_attn_gpu import BF16_REL_L2, reference_attention, rel_l2

    rows, heads = 500, 3
    g = torch.Generator(device=dev).manual_seed(7)
    q, k, v = (torch.randn(1, rows * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    sl = slice(rank * rows, (rank + 1) * rows)
    ring = RingAttention(world=world, rank=rank, batch=1, q_len=rows, kv_len=rows, heads=heads,
                         kv_heads=heads, head_dim=128, device=dev, generation=2)
    # Several calls back to back with different inputs and no host sync in
    # between: the closing barrier keeps a call's first rotation from
    # overwriting a block a neighbour still attends in the previous call.
    calls = []
    for n in range(4):
        qn, kn, vn = (t * (1.0 + 0.25 * n) for t in (q, k, v))
        lse = torch.empty(1, heads, rows, device=dev, dtype=torch.float32)
        out, _ = ring.forward(qn[:, sl].contiguous(), kn[:, sl].contiguous(), vn[:, sl].contiguous(), lse=lse)
        calls.append((qn, kn, vn, out, lse))
    torch.cuda.synchronize()
    for n, (qn, kn, vn, out, lse) in enumerate(calls):
        ref, ref_lse = reference_attention(qn, kn, vn)
        check.le(rel_l2(out, ref[:, sl]), BF16_REL_L2, f"ring call {n} rel l2")
        check.le((lse - ref_lse[:, :, sl]).abs().max().item(), 2e-3, f"ring call {n} lse")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    ring.close()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_ring_across_gpus_matches_unsharded_attention():
    _spawn(_ring_case, min(torch.cuda.device_count(), 4))


def _per_block_e4m3(t, world):
    """(e4m3 blocks, descales, the dequantized whole axis) of a (1, world*L, H, D)
    tensor cut into `world` row blocks, each quantised over its own rows."""
    from tests.test_attn_gpu import quantize_e4m3_per_head

    blocks = t.chunk(world, dim=1)
    quant = [quantize_e4m3_per_head(b) for b in blocks]
    deq = torch.cat([x.float() * sc.view(1, 1, -1, 1) for x, sc in quant], dim=1)
    return quant, deq


def _ring_fp8_case(rank, world, dev):
    """e4m3 ring: every rank quantises its query rows and its K/V block with
    per-head scales over those rows; the blocks rotate with their descales.
    Held to fp32 attention over the per-block dequantized axis."""
    check = Checks(rank)
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ring import RingAttention
    from tests.test_attn_gpu import FP8_REL_L2, reference_attention, rel_l2

    rows, heads = 500, 3
    g = torch.Generator(device=dev).manual_seed(8)
    q, k, v = (torch.randn(1, rows * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    (qq, qd), (kq, kd), (vq, vd) = (_per_block_e4m3(t, world) for t in (q, k, v))
    ring = RingAttention(world=world, rank=rank, batch=1, q_len=rows, kv_len=rows, heads=heads,
                         kv_heads=heads, head_dim=128, device=dev, generation=3, dtype=torch.float8_e4m3fn)
    for n in range(2):
        lse = torch.empty(1, heads, rows, device=dev, dtype=torch.float32)
        out, _ = ring.forward(qq[rank][0], kq[rank][0], vq[rank][0], lse=lse, q_descale=qq[rank][1],
                              k_descale=kq[rank][1], v_descale=vq[rank][1])
        torch.cuda.synchronize()
        sl = slice(rank * rows, (rank + 1) * rows)
        ref, ref_lse = reference_attention(qd[:, sl], kd, vd)
        check(out.dtype == torch.bfloat16, f"output dtype {out.dtype}")
        check.le(rel_l2(out, ref), FP8_REL_L2, f"fp8 ring call {n} rel l2")
        check.le((lse - ref_lse).abs().max().item(), 5e-3, f"fp8 ring call {n} lse")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    ring.close()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_fp8_ring_across_gpus_with_per_block_scales():
    _spawn(_ring_fp8_case, min(torch.cuda.device_count(), 4))


def _usp_fp8_ring_case(rank, world, dev):
    """The FP8 drop-in over a pure ring group: each rank's rows and block are
    quantised where they live, as the reference's ring loop hands an inner FP8
    kernel one block at a time."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.usp import make_b200_usp_attention
    from tests.test_attn_gpu import FP8_REL_L2, reference_attention, rel_l2

    check = Checks(rank)
    attn = make_b200_usp_attention(ring_group=dist_world_group(), generation=43, device=dev, fp8=True)
    heads, ls = 4, 384
    g = torch.Generator(device=dev).manual_seed(79)
    q, k, v = (torch.randn(1, ls * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    rows = slice(rank * ls, (rank + 1) * ls)
    (_, qd), (_, kd), (_, vd) = (_per_block_e4m3(t, world) for t in (q, k, v))
    out = attn(*(t[:, rows].reshape(1, ls, -1) for t in (q, k, v)), heads=heads)
    torch.cuda.synchronize()
    ref, _ = reference_attention(qd[:, rows], kd, vd)
    check.le(rel_l2(out.reshape(1, ls, heads, 128), ref), FP8_REL_L2, "fp8 ring drop-in rel l2")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    attn.impl.invalidate()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_fp8_drop_in_over_a_ring_group():
    _spawn(_usp_fp8_ring_case, min(torch.cuda.device_count(), 4))


def _usp_gqa_ring_case(rank, world, dev):
    """GQA over a ring group: the ring rotates the shared K/V heads alone (no
    expansion), and the result equals attention with K/V repeated per group."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.usp import make_b200_usp_attention
    from tests.test_attn_gpu import BF16_REL_L2, reference_attention, rel_l2

    check = Checks(rank)
    attn = make_b200_usp_attention(ring_group=dist_world_group(), generation=44, device=dev)
    heads, kv_heads, ls = 4, 2, 320
    g = torch.Generator(device=dev).manual_seed(81)
    q = torch.randn(1, ls * world, heads, 128, device=dev, generator=g).bfloat16()
    k, v = (torch.randn(1, ls * world, kv_heads, 128, device=dev, generator=g).bfloat16() for _ in range(2))
    rows = slice(rank * ls, (rank + 1) * ls)
    out = attn(q[:, rows].reshape(1, ls, -1), k[:, rows].reshape(1, ls, -1), v[:, rows].reshape(1, ls, -1),
               heads=heads, enable_gqa=True)
    torch.cuda.synchronize()
    ref, _ = reference_attention(q, k.repeat_interleave(2, dim=2), v.repeat_interleave(2, dim=2))
    check.le(rel_l2(out.reshape(1, ls, heads, 128), ref[:, rows]), BF16_REL_L2, "gqa ring rel l2")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    attn.impl.invalidate()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_gqa_drop_in_over_a_ring_group_without_expansion():
    _spawn(_usp_gqa_ring_case, min(torch.cuda.device_count(), 4))


def dist_world_group():
    import torch.distributed as dist

    return dist.group.WORLD


def _callable_case(rank, world, dev):
    """The drop-in usp_attention on a Ulysses group: plain, joint order with
    pad rows, and native GQA, against unsharded attention."""
    check = Checks(rank)
    import torch.distributed as dist

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.usp import make_b200_usp_attention
    from oracle import usp as oracle_usp
    from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, reference_attention, rel_l2

    group = dist.new_group(list(range(world)))
    attn = make_b200_usp_attention(ulysses_group=group, generation=3, device=dev)
    heads, d = 2 * world, 128
    # 1) plain Ulysses, comfy (B, L, H*D) layout
    ls = 256
    g = torch.Generator(device=dev).manual_seed(31)
    q, k, v = (torch.randn(1, ls * world, heads, d, device=dev, generator=g).bfloat16() for _ in range(3))
    sl = slice(rank * ls, (rank + 1) * ls)
    out = attn(*(t[:, sl].reshape(1, ls, -1) for t in (q, k, v)), heads=heads)
    ref, _ = reference_attention(q, k, v)
    check.le(rel_l2(out.reshape(1, ls, heads, d), ref[:, sl]), BF16_REL_L2, "plain rel l2")
    # 2) joint [text, image] order with one image pad row on the last rank
    text, image = 32, 96
    ls2 = text + image
    txt = [torch.randn(1, text * world, heads, d, device=dev, generator=g).bfloat16() for _ in range(3)]
    img = [torch.randn(1, image * world, heads, d, device=dev, generator=g).bfloat16() for _ in range(3)]
    for t in img:
        t[:, -1] = 0  # the synthetic pad shard_seq appends
    local = [torch.cat((tt[:, rank * text:(rank + 1) * text], ii[:, rank * image:(rank + 1) * image]), dim=1)
             for tt, ii in zip(txt, img)]
    pad = [(world - 1) * ls2 + ls2 - 1]  # rank-major coordinate of the last image row
    order = oracle_usp.RankMajorJointOrder(text, image)
    out2 = attn(*(t.transpose(1, 2) for t in local), heads=heads, skip_reshape=True,
                skip_output_reshape=True, drop_rows=pad, sequence_order=order).transpose(1, 2)
    full = [torch.cat((tt, ii[:, :-1]), dim=1) for tt, ii in zip(txt, img)]  # stock order, pad dropped
    ref2, _ = reference_attention(*full)
    want_txt = ref2[:, rank * text:(rank + 1) * text]
    img_rows = ref2[:, text * world:]
    want_img = img_rows[:, rank * image:(rank + 1) * image]
    got_img = out2[:, text:]
    if rank == world - 1:
        check(torch.equal(got_img[:, -1], torch.zeros_like(got_img[:, -1])), "joint pad row not zero")
        got_img = got_img[:, :-1]
    check.le((out2[:, :text].float() - want_txt).abs().max().item(), BF16_MAX_ABS, "joint text max abs")
    check.le((got_img.float() - want_img).abs().max().item(), BF16_MAX_ABS, "joint image max abs")
    # 3) native GQA: K/V heads split by the Ulysses degree
    hkv = world
    qg = torch.randn(1, ls * world, heads, d, device=dev, generator=g).bfloat16()
    kg, vg = (torch.randn(1, ls * world, hkv, d, device=dev, generator=g).bfloat16() for _ in range(2))
    out3 = attn(qg[:, sl].reshape(1, ls, -1), kg[:, sl].reshape(1, ls, -1), vg[:, sl].reshape(1, ls, -1),
                heads=heads, enable_gqa=True)
    ref3, _ = reference_attention(qg, kg, vg)
    check.le(rel_l2(out3.reshape(1, ls, heads, d), ref3[:, sl]), BF16_REL_L2, "gqa rel l2")
    # 4) LTX guide biases plus a per-head key bias on a stream with tail pads:
    #    the kernel applies the groups on the gathered axis and routes rows home
    from tests.test_usp_callable_gpu import ltx_guide_groups, oracle_grouped

    real = ls * world - 9
    qb, kb, vb = (torch.randn(1, ls * world, heads, d, device=dev, generator=g).bfloat16() for _ in range(3))
    weights = torch.rand(100, device=dev, generator=g) + 0.05
    weights[3] = 0.0
    groups = ltx_guide_groups(real, real - 180, weights)
    groups[-1] = (groups[-1][0], groups[-1][1], torch.randn(1, heads, 1, real, device=dev, generator=g))
    drop = list(range(real, ls * world))
    out4 = attn(*(t[:, sl].transpose(1, 2) for t in (qb, kb, vb)), heads=heads, skip_reshape=True,
                skip_output_reshape=True, drop_rows=drop, query_bias_groups=groups).transpose(1, 2)
    want4 = oracle_grouped(qb, kb, vb, drop, groups)[:, sl]
    check.le((out4.double() - want4).abs().max().item(), BF16_MAX_ABS, "bias groups max abs")
    torch.cuda.synchronize()
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    attn.impl.invalidate()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_usp_callable_across_gpus():
    _spawn(_callable_case, min(torch.cuda.device_count(), 4))


def _cfg_fp8_case(rank, world, dev):
    """CFG split across GPUs with FP8 attention (the C3 shape family, small):
    batch 2 (cond, uncond) -> one row per cfg rank -> e4m3 attention ->
    peer-store all-gather of the predictions, in rank order."""
    check = Checks(rank)
    import torch.distributed as dist

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.cfg import CfgGather, cfg_parallel_call
    from dgx_monarch_b200.usp import make_b200_usp_attention
    from tests.test_attn_gpu import reference_attention, rel_l2

    cfg_group = dist.new_group(list(range(world)))
    attn = make_b200_usp_attention(generation=4, device=dev, fp8=True)  # Ulysses degree 1 per cfg rank
    batch, l, heads = world, 640, 4
    g = torch.Generator(device=dev).manual_seed(53)
    x = torch.randn(batch, l, 3, heads, 128, device=dev, generator=g).bfloat16()

    def forward(x):
        q, k, v = (x[:, :, i].reshape(x.shape[0], l, -1) for i in range(3))
        return attn(q, k, v, heads=heads)

    gather = CfgGather(l * heads * 128 * 2, device=dev, group=cfg_group, generation=4)
    full = cfg_parallel_call(forward, x, group=cfg_group, gather=gather).reshape(batch, l, heads, 128)
    torch.cuda.synchronize()
    from tests.test_attn_gpu import FP8_REL_L2, fp8_references

    ref, _ = reference_attention(x[:, :, 0], x[:, :, 1], x[:, :, 2])
    check(full.shape == (batch, l, heads, 128), f"gathered shape {tuple(full.shape)}")
    for bi in range(batch):
        # each cfg rank quantises its own batch row
        ref_deq, floor = fp8_references(*(x[bi:bi + 1, :, i] for i in range(3)))
        check.le(rel_l2(full[bi], ref_deq[0]), FP8_REL_L2, f"cfg row {bi} rel l2 vs its e4m3 inputs")
        check.le(rel_l2(full[bi], ref[bi]), floor + FP8_REL_L2, f"cfg row {bi} rel l2 vs activations")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    gather.close()
    attn.impl.invalidate()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_cfg_split_fp8_across_gpus():
    _spawn(_cfg_fp8_case, 2)


def _full_context_case(rank, world, dev):
    """The Wan Ring2 full-context path (adapters/wan_ring_full_context.py):
    the class at any ring degree, then the reference-signature function and
    the drop-in's full_context_ring option at ring degree 2."""
    import torch.distributed as dist

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ring import FullContextRingAttention
    from dgx_monarch_b200.usp import UnsupportedModelError, make_b200_usp_attention
    from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, LSE_ABS, reference_attention, rel_l2

    check = Checks(rank)
    rows, heads = 300, 3
    g = torch.Generator(device=dev).manual_seed(61)
    q, k, v = (torch.randn(2, rows * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    sl = slice(rank * rows, (rank + 1) * rows)
    ref, ref_lse = reference_attention(q, k, v)
    fc = FullContextRingAttention(world=world, rank=rank, batch=2, q_len=rows, kv_len=rows, heads=heads,
                                  kv_heads=heads, head_dim=128, device=dev, generation=8)
    lse = torch.empty(2, heads, rows, device=dev, dtype=torch.float32)
    for step in range(3):  # alternating window buffers
        ql, kl, vl = (t[:, sl].contiguous() for t in (q, k, v))
        if step == 2:  # strided views of a packed layout are gathered as well
            packed = torch.stack((q[:, sl], k[:, sl], v[:, sl]), dim=2)
            ql, kl, vl = packed[:, :, 0], packed[:, :, 1], packed[:, :, 2]
        out, _ = fc.forward(ql, kl, vl, lse=lse)
        torch.cuda.synchronize()
        check.le((out.float() - ref[:, sl]).abs().max().item(), BF16_MAX_ABS, f"class step {step} max abs")
        check.le(rel_l2(out, ref[:, sl]), BF16_REL_L2, f"class step {step} rel l2")
        check.le((lse - ref_lse[:, :, sl]).abs().max().item(), LSE_ABS, f"class step {step} lse")
    fc.close()
    if world == 2:
        from dgx_monarch_b200.full_context import make_full_context_ring_attention

        group = dist.new_group([0, 1])
        fn = make_full_context_ring_attention(ring_group=group, generation=9, device=dev)
        ql, kl, vl = (t[:, sl].contiguous() for t in (q, k, v))
        refused = 0
        for kwargs in ({"causal": True}, {"dropout_p": 0.1}, {"window_size": (4, 4)},
                       {"softmax_scale": 0.5}, {"q_descale": torch.ones(1)}):
            try:
                fn(ql, kl, vl, **kwargs)
            except UnsupportedModelError:
                refused += 1
        check(refused == 5, f"{refused} of 5 unsupported surfaces refused")
        # fp16 shards run in fp16, as the reference's flash path takes them
        # (adapters/wan_ring_full_context.py:10), and are held to the fp16 bound.
        from tests.test_attn_gpu import F16_REL_L2

        out16 = fn(ql.half(), kl.half(), vl.half())
        ref16, _ = reference_attention(q.half(), k.half(), v.half())
        check(out16.dtype == torch.float16, f"fp16 shards gave {out16.dtype}")
        check.le(rel_l2(out16, ref16[:, sl]), F16_REL_L2, "fp16 reference-signature function rel l2")
        out = fn(ql, kl, vl, group=group)
        check.le(rel_l2(out, ref[:, sl]), BF16_REL_L2, "reference-signature function rel l2")
        fn.invalidate()
        attn = make_b200_usp_attention(ring_group=group, generation=10, device=dev, full_context_ring=True)
        out = attn(*(t.reshape(2, rows, -1) for t in (ql, kl, vl)), heads=heads)
        check.le(rel_l2(out.reshape(2, rows, heads, 128), ref[:, sl]), BF16_REL_L2, "drop-in rel l2")
        attn.impl.invalidate()
    torch.cuda.synchronize()
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_full_context_ring_across_gpus():
    _spawn(_full_context_case, 2)
    if torch.cuda.device_count() >= 4:
        _spawn(_full_context_case, 4)


def _shard_case(rank, world, dev):
    """sp_gather over NVLink (adapters/base.py:126-131) and the shared NVFP4
    activation scale (adapters/quant_activation_scale.py:222-246)."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.shard import NVFP4_SCALE_DIVISOR, SequenceGather, SharedActivationScale, shard_seq

    check = Checks(rank)
    gather = SequenceGather(device=dev, generation=12)
    g = torch.Generator(device=dev).manual_seed(71)
    cases = [
        torch.randn(2, 1001, 3072, device=dev, generator=g).bfloat16(),  # pads on the last rank
        torch.randn(1, 4, 37, 128, device=dev, generator=g),            # fp32, gathered on dim 2
        torch.randn(3, 50, 3, device=dev, generator=g).half(),           # 6-byte rows
        torch.randn(2, 1001, 3072, device=dev, generator=g).bfloat16(),  # the first shape again
    ]
    for n, x in enumerate(cases):
        dim = 2 if x.ndim == 4 else 1
        local, orig = shard_seq(x, world, rank, dim=dim)
        got = gather(local, orig, dim=dim)
        torch.cuda.synchronize()
        check(got.shape == x.shape and torch.equal(got, x), f"sp_gather case {n} differs")
    gather.close()

    scale = SharedActivationScale(device=dev, generation=13)
    for n, (dtype, rows, cols) in enumerate(((torch.bfloat16, 256, 3072), (torch.float16, 64, 40),
                                             (torch.float32, 96, 520), (torch.bfloat16, 8, 7))):
        x = torch.randn(rows, cols, device=dev, generator=g).to(dtype)
        x[rows - 1, cols // 2] = 37.5  # the outlier sits on the last rank's rows
        local, _ = shard_seq(x, world, rank, dim=0)
        trace: list = []
        got = scale(local, trace=trace)
        want = x.abs().amax().to(torch.float32).reshape(()).to(dtype) / NVFP4_SCALE_DIVISOR
        torch.cuda.synchronize()
        check(got.dtype == dtype and torch.equal(got, want), f"scale case {n}: {got.item()} vs {want.item()}")
        check(trace[1].item() == 37.5, f"reduced amax case {n}: {trace[1].item()}")
    nan = torch.zeros(4, 16, device=dev, dtype=torch.bfloat16)
    if rank == 0:
        nan[1, 3] = float("nan")
    got = scale(nan)
    torch.cuda.synchronize()
    check(torch.isnan(got).item(), "a NaN on one rank must reach every rank's scale")
    scale.close()
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_sequence_gather_and_shared_scale_across_gpus():
    _spawn(_shard_case, min(torch.cuda.device_count(), 4))


def _dual_cfg_case(rank, world, dev):
    """dm-cfg2 (actor/dual_model_cfg.py:75-94): rank 0 holds the conditional
    prediction, rank 1 the unconditional; both must end with the identical
    combined prediction, step after step."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.cfg import DualModelCfg

    check = Checks(rank)
    shape = (1, 16, 128, 128)
    split = DualModelCfg(math.prod(shape) * 4, 4.0, device=dev, generation=14)
    for step in range(3):  # alternating window buffers
        g = torch.Generator(device=dev).manual_seed(80 + step)
        cond = torch.randn(shape, device=dev, generator=g)
        uncond = torch.randn(shape, device=dev, generator=g)
        got = split(cond if rank == 0 else uncond)
        torch.cuda.synchronize()
        check(torch.equal(got, uncond + (cond - uncond) * 4.0), f"step {step}: combined prediction differs")
    split.close()
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_dual_model_cfg_split_across_gpus():
    _spawn(_dual_cfg_case, 2)


def _cond_dispatch_case(rank, world, dev):
    """Per-conditioning CFG dispatch (adapters/cfg_dispatch.py:209-271) over
    real cfg ranks: conditionings that do not batch (7, 11 and 13 text tokens)
    are spread over the ranks, each rank runs only its group, and the
    NVLink gather hands every rank the one-GPU output list in cond order,
    call after call."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.cfg import CfgGather
    from dgx_monarch_b200.cfg_dispatch import CondDispatch

    class Tokens:
        def __init__(self, n):
            self.cond = torch.zeros(1, n, 4)

        def process_cond(self, batch_size, area):
            return self

        def can_concat(self, other):
            a, b = sorted((self.cond.shape[1], other.cond.shape[1]))
            return a == b or (a > 0 and math.lcm(a, b) // a <= 4)

    def executor(conds, x):
        out = [torch.zeros_like(x) for _ in conds]
        for i, slot in enumerate(conds):
            for item in slot or []:
                out[i] = out[i] + x * item["weight"] + float(item["model_conds"]["c"].cond.shape[1])
        return out

    check = Checks(rank)
    conds = [[{"model_conds": {"c": Tokens(n)}, "weight": float(w)}] for n, w in ((7, 2), (11, 5), (13, 9))]
    x = torch.arange(2 * 16 * 64 * 64, device=dev, dtype=torch.float32).reshape(2, 16, 64, 64) / 1e5
    size = -(-len(conds) // world)
    gather = CfgGather(size * x.numel() * x.element_size(), device=dev, generation=23)
    dispatch = CondDispatch(world=world, rank=rank, gather=gather)
    for step in range(3):
        xs = x + step
        got = dispatch(executor, conds, xs)
        want = executor(conds, xs)
        torch.cuda.synchronize()
        check(dispatch.last_path == "dispatch", f"path {dispatch.last_path}")
        check(len(got) == 3 and all(torch.equal(a, b) for a, b in zip(got, want)),
              f"call {step}: the gathered outputs differ from the one-GPU list")
    gather.close()
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_per_cond_cfg_dispatch_across_gpus():
    _spawn(_cond_dispatch_case, 2)


def _graph_case(rank, world, dev):
    """A Ulysses step (scatter, barrier, routed attention, barrier) captured in
    a CUDA graph and replayed with new inputs: the barrier epochs advance on
    the device, so every replay synchronises afresh."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ulysses import UlyssesAttention
    from tests.test_attn_gpu import BF16_REL_L2, reference_attention, rel_l2

    check = Checks(rank)
    heads, ls = 2 * world, 256
    uly = UlyssesAttention(world=world, rank=rank, batch=1, seq_local=ls, heads=heads, head_dim=128,
                           device=dev, generation=15)
    bufs = [torch.zeros(1, ls, heads, 128, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    out = torch.zeros(1, ls, heads, 128, device=dev, dtype=torch.bfloat16)
    uly.forward(*bufs)  # warm-up outside the capture (kernel attributes, plans)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out.copy_(uly.forward(*bufs))
    for step in range(3):
        g = torch.Generator(device=dev).manual_seed(90 + step)  # the same full tensors on every rank
        q, k, v = (torch.randn(1, ls * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
        for buf, full in zip(bufs, (q, k, v)):
            buf.copy_(full[:, rank * ls:(rank + 1) * ls])
        graph.replay()
        torch.cuda.synchronize()
        ref, _ = reference_attention(q, k, v)
        check.le(rel_l2(out, ref[:, rank * ls:(rank + 1) * ls]), BF16_REL_L2, f"replay {step} rel l2")
    del graph
    uly.close()
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_captured_ulysses_step_replays_across_gpus():
    _spawn(_graph_case, 2)


def _streamed_case(rank, world, dev):
    """Ulysses attention over pinned host tensors streamed by head groups, each
    group its own Ulysses step, against unsharded attention."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ulysses import HostStreamedUlysses
    from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, reference_attention, rel_l2

    check = Checks(rank)
    heads, ls = 4 * world, 300
    g = torch.Generator(device=dev).manual_seed(97)
    q, k, v = (torch.randn(1, ls * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    sl = slice(rank * ls, (rank + 1) * ls)
    hq, hk, hv = (t[:, sl].contiguous().cpu().pin_memory() for t in (q, k, v))
    hout = torch.full((1, ls, heads, 128), float("nan"), dtype=torch.bfloat16).pin_memory()
    streamed = HostStreamedUlysses(world=world, rank=rank, batch=1, seq_local=ls, heads=heads, head_dim=128,
                                   device=dev, groups=2, generation=16)
    ref, _ = reference_attention(q, k, v)
    for step in range(2):
        streamed(hq, hk, hv, hout)
        torch.cuda.synchronize()
        got = hout.to(dev)
        check.le((got.float() - ref[:, sl]).abs().max().item(), BF16_MAX_ABS, f"call {step} max abs")
        check.le(rel_l2(got, ref[:, sl]), BF16_REL_L2, f"call {step} rel l2")
    streamed.close()
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_host_streamed_ulysses_across_gpus():
    _spawn(_streamed_case, 2)


def _peer_timeout_case(rank, world, dev):
    """Failure detection without a GPU fault: rank 1 never arrives at a
    barrier (the failure is made on the host), rank 0's barrier kernel gives up
    after its 200 ms budget, sets the peer-timeout bit of the device error word
    and returns, and the context stays usable for the next kernel."""
    import torch.distributed as dist

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.comm import PeerWindows
    from dgx_monarch_b200.ops import attention_fwd
    from tests.test_attn_gpu import BF16_REL_L2, reference_attention, rel_l2

    check = Checks(rank)
    win = PeerWindows(1 << 20, device=dev, rank=rank, world=world, generation=18)
    win.set_timeout(200)
    win.barrier()                      # both ranks: a barrier that completes
    torch.cuda.synchronize()
    check(_lib.device_error() == 0, "the completed barrier reported an error")
    dist.barrier()
    if rank == 0:
        win.barrier()                  # rank 1 never arrives at this one
        torch.cuda.synchronize()
        word = _lib.device_error()     # read and clear
        check(word & _lib.ERR_PEER_TIMEOUT != 0, f"device error word {word} lacks the peer-timeout bit")
        g = torch.Generator(device=dev).manual_seed(3)
        q, k, v = (torch.randn(1, 300, 2, 128, device=dev, generator=g).bfloat16() for _ in range(3))
        out, _ = attention_fwd(q, k, v, return_lse=False)
        ref, _ = reference_attention(q, k, v)
        torch.cuda.synchronize()
        check.le(rel_l2(out, ref), BF16_REL_L2, "attention after the expired wait")
        check(_lib.device_error() == 0, "the context reported errors after recovery")
    dist.barrier()                     # the host learns of the missing rank; both retire the windows
    win.close()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_expired_barrier_reports_and_the_context_recovers():
    _spawn(_peer_timeout_case, 2)


def _overlapped_case(rank, world, dev):
    """The overlapped Ulysses step (group scatters hidden behind attention,
    two receive slots) gives the same bits as the plain step, call after call."""
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ulysses import OverlappedUlysses, UlyssesAttention

    check = Checks(rank)
    heads, ls = 4 * world, 300
    plain = UlyssesAttention(world=world, rank=rank, batch=1, seq_local=ls, heads=heads, head_dim=128,
                             device=dev, generation=19)
    for n, groups in enumerate((4, 2, [world, 3 * world], [world, world, 2 * world])):
        over = OverlappedUlysses(world=world, rank=rank, batch=1, seq_local=ls, heads=heads, head_dim=128,
                                 device=dev, groups=groups, generation=20 + n)
        for step in range(3):
            g = torch.Generator(device=dev).manual_seed(110 + step + rank)
            q, k, v = (torch.randn(1, ls, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
            want = plain.forward(q, k, v).clone()
            got = over.forward(q, k, v).clone()
            torch.cuda.synchronize()
            check(torch.equal(got, want), f"{groups} groups, call {step}: differs from the plain step")
        over.close()
    plain.close()
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_overlapped_ulysses_equals_plain_step():
    _spawn(_overlapped_case, min(torch.cuda.device_count(), 4))


def _joint_case(rank, world, dev):
    """Joint image+text attention with the text replicated: 1024 image rows
    split by sequence, 256 text rows on every rank, 8 heads of 64, fp32 in and
    out.  Every rank's text output is the same bytes; both outputs are the
    one-rank result bit for bit, and within the bf16 bound of fp32 attention
    over the unsharded [text | image] concatenation."""
    import torch.distributed as dist

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ulysses import JointUlyssesAttention
    from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, reference_attention, rel_l2

    check = Checks(rank)
    heads, d, image, text = 8, 64, 1024, 256
    ls = image // world
    g = torch.Generator(device=dev).manual_seed(2024)
    img = [torch.randn(1, image, heads, d, device=dev, generator=g) for _ in range(3)]
    txt = [torch.randn(1, text, heads, d, device=dev, generator=g) for _ in range(3)]
    mine = [x[:, rank * ls:(rank + 1) * ls].contiguous() for x in img]
    for text_first in (True, False):
        joint = JointUlyssesAttention(world=world, rank=rank, batch=1, seq_local=ls, txt_rows=text,
                                      heads=heads, head_dim=d, device=dev, text_first=text_first,
                                      generation=31 + int(text_first))
        out_img, out_txt = joint(*mine, *txt)
        torch.cuda.synchronize()
        joint.close()
        alone = JointUlyssesAttention(world=1, rank=0, batch=1, seq_local=image, txt_rows=text, heads=heads,
                                      head_dim=d, device=dev, text_first=text_first)
        one_img, one_txt = alone(*img, *txt)
        torch.cuda.synchronize()
        alone.close()
        tag = "text first" if text_first else "text last"
        check(out_img.dtype == torch.float32 and out_txt.dtype == torch.float32, f"{tag}: output dtype")
        check(torch.equal(out_img, one_img[:, rank * ls:(rank + 1) * ls]), f"{tag}: image rows differ from one rank")
        check(torch.equal(out_txt, one_txt), f"{tag}: text differs from one rank")
        every = [torch.empty_like(out_txt) for _ in range(world)]
        dist.all_gather(every, out_txt)
        check(all(torch.equal(e, every[0]) for e in every), f"{tag}: ranks hold different text outputs")
        q, k, v = (torch.cat([a, b] if text_first else [b, a], dim=1).bfloat16() for a, b in zip(txt, img))
        ref, _ = reference_attention(q, k, v)
        ref_txt, ref_img = (ref[:, :text], ref[:, text:]) if text_first else (ref[:, image:], ref[:, :image])
        for got, want, what in ((out_img, ref_img[:, rank * ls:(rank + 1) * ls], "image"), (out_txt, ref_txt, "text")):
            check.le((got - want).abs().max().item(), BF16_MAX_ABS, f"{tag}: {what} max-abs")
            check.le(rel_l2(got, want), BF16_REL_L2, f"{tag}: {what} rel-L2")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_joint_attention_with_replicated_text_across_gpus():
    _spawn(_joint_case, 2)
    if torch.cuda.device_count() >= 4:
        _spawn(_joint_case, 4)


def _hybrid_case(rank, world, dev):
    """Ulysses inside runs of consecutive ranks and ring across them (the
    ulysses-low layout of oracle.usp.hybrid_groups): each rank holds one
    sequence chunk in rank order, and its output rows equal unsharded
    attention over the whole sequence."""
    import torch.distributed as dist

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.usp import make_b200_usp_attention
    from oracle.usp import hybrid_groups
    from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, reference_attention, rel_l2

    check = Checks(rank)
    uly, ring = 2, world // 2
    ulysses_groups, ring_groups = hybrid_groups(world, uly, ring)
    mine_u = mine_r = None
    for ranks in ulysses_groups:
        grp = dist.new_group(ranks)
        if rank in ranks:
            mine_u = grp
    for ranks in ring_groups:
        grp = dist.new_group(ranks)
        if rank in ranks:
            mine_r = grp
    attn = make_b200_usp_attention(ulysses_group=mine_u, ring_group=mine_r, generation=41, device=dev)
    heads, ls = 4, 300
    g = torch.Generator(device=dev).manual_seed(77)
    q, k, v = (torch.randn(1, ls * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    rows = slice(rank * ls, (rank + 1) * ls)
    for step in range(2):
        out = attn(*(t[:, rows].reshape(1, ls, -1) for t in (q, k, v)), heads=heads)
        torch.cuda.synchronize()
        ref, _ = reference_attention(q, k, v)
        got = out.reshape(1, ls, heads, 128)
        check.le((got.float() - ref[:, rows]).abs().max().item(), BF16_MAX_ABS, f"call {step} max abs")
        check.le(rel_l2(got, ref[:, rows]), BF16_REL_L2, f"call {step} rel l2")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    attn.impl.invalidate()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four or more GPUs")
def test_hybrid_ulysses_ring_across_gpus():
    _spawn(_hybrid_case, 4)


def _hybrid_fp8_case(rank, world, dev):
    """FP8 over Ulysses-2 x ring-2 (ulysses-low): after the scatter a rank holds
    its Ulysses group's rows (half the sequence) for half the heads, quantises
    them per head and rotates its K/V block with its scales.  So q, k and v are
    quantised per head over each half of the sequence; held to fp32 attention
    over those dequantized halves."""
    import torch.distributed as dist

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.groups import hybrid_layout
    from dgx_monarch_b200.usp import make_b200_usp_attention
    from tests.test_attn_gpu import FP8_REL_L2, reference_attention, rel_l2

    check = Checks(rank)
    uly, ring = 2, world // 2
    ulysses_groups, ring_groups = hybrid_layout(world, uly, ring)
    mine_u = mine_r = None
    for ranks in ulysses_groups:
        grp = dist.new_group(ranks)
        if rank in ranks:
            mine_u = grp
    for ranks in ring_groups:
        grp = dist.new_group(ranks)
        if rank in ranks:
            mine_r = grp
    attn = make_b200_usp_attention(ulysses_group=mine_u, ring_group=mine_r, generation=45, device=dev, fp8=True)
    heads, ls = 4, 256
    g = torch.Generator(device=dev).manual_seed(83)
    q, k, v = (torch.randn(1, ls * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    rows = slice(rank * ls, (rank + 1) * ls)
    (_, qd), (_, kd), (_, vd) = (_per_block_e4m3(t, ring) for t in (q, k, v))
    out = attn(*(t[:, rows].reshape(1, ls, -1) for t in (q, k, v)), heads=heads)
    torch.cuda.synchronize()
    ref, _ = reference_attention(qd, kd, vd)
    check.le(rel_l2(out.reshape(1, ls, heads, 128), ref[:, rows]), FP8_REL_L2, "hybrid fp8 rel l2")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    attn.impl.invalidate()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four or more GPUs")
def test_hybrid_ulysses_ring_fp8_across_gpus():
    _spawn(_hybrid_fp8_case, 4)
