"""The allocation-free ring attention entry point (dgxm_ring_attn_fwd_noalloc).

Some callers cannot call cudaMalloc when attention runs -- their device memory
belongs to another allocator with a fixed budget, or cudaMalloc would stall
the device on a latency-critical path.  This entry point keeps the ring's
partial results in a static array of module memory instead of a workspace.
The test calls it through the C ABI twice in a row and checks each result
against the workspace entry point's, within the bf16 tolerance of the other
attention tests.  Ring attention needs at least two GPUs (one rank each).

This file is collected last, so a run that stops at the first failure has
already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from tests.test_multigpu import Checks, _spawn

pytestmark = pytest.mark.gpu


def _noalloc_case(rank, world, dev):
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ops import attn_desc
    from dgx_monarch_b200.ring import RingAttention
    from tests.test_attn_gpu import BF16_MAX_ABS, BF16_REL_L2, LSE_ABS, reference_attention, rel_l2

    check = Checks(rank)
    lib = _lib.load()
    rows, heads = 384, 4
    g = torch.Generator(device=dev).manual_seed(101)
    q, k, v = (torch.randn(1, rows * world, heads, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    sl = slice(rank * rows, (rank + 1) * rows)
    ql, kl, vl = (t[:, sl].contiguous() for t in (q, k, v))
    ring = RingAttention(world=world, rank=rank, batch=1, q_len=rows, kv_len=rows, heads=heads,
                         kv_heads=heads, head_dim=128, device=dev, generation=21)
    want = torch.empty(1, rows, heads, 128, device=dev, dtype=torch.bfloat16)
    want_lse = torch.empty(1, heads, rows, device=dev, dtype=torch.float32)
    ring.forward(ql, kl, vl, out=want, lse=want_lse)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(2):  # two calls in a row: the shared array keeps the last call's contents
        got = torch.full_like(want, float("nan"))
        got_lse = torch.full_like(want_lse, float("nan"))
        desc = attn_desc(ql, kl, vl, got, got_lse)
        rc = lib.dgxm_ring_attn_fwd_noalloc(ring.windows._handle, ctypes.byref(desc), ql.data_ptr(),
                                            kl.data_ptr(), vl.data_ptr(), got.data_ptr(),
                                            got_lse.data_ptr(), stream)
        check(rc == 0, f"dgxm_ring_attn_fwd_noalloc returned {rc}")
        torch.cuda.synchronize(dev)
        check.le((got.float() - want.float()).abs().max().item(), BF16_MAX_ABS, "max abs vs workspace entry")
        check.le(rel_l2(got, want), BF16_REL_L2, "rel l2 vs workspace entry")
        check.le((got_lse - want_lse).abs().max().item(), LSE_ABS, "lse vs workspace entry")
    ref, _ = reference_attention(q, k, v)
    check.le(rel_l2(got, ref[:, sl]), BF16_REL_L2, "rel l2 vs unsharded attention")
    # A shape whose partial results exceed the static array is refused, not truncated.
    big_q = torch.empty(1, 1 << 20, heads, 128, device="meta", dtype=torch.bfloat16)
    desc = attn_desc(big_q, kl, vl, big_q, None)
    rc = lib.dgxm_ring_attn_fwd_noalloc(ring.windows._handle, ctypes.byref(desc), None, None, None,
                                        None, None, stream)
    check(rc == _lib.DGXM_ERR_INVALID, f"oversized shape returned {rc}")
    check(b"32 MiB" in lib.dgxm_last_error_message(), "refusal names the 32 MiB limit")
    check(lib.dgxm_ring_noalloc_max_bytes() == 32 << 20, "static array size")
    check(_lib.device_error() == 0, f"device error word {_lib.device_error()}")
    ring.close()
    check.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="ring attention needs two or more GPUs")
def test_noalloc_ring_matches_workspace_ring_twice():
    _spawn(_noalloc_case, 2)
