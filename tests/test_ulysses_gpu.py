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
