"""World-size-2 gloo tests on CPU.

C1: Ulysses joint attention in fp32, B=1, 1024 image + 256 text tokens, H=8,
D=64, Q/K/V ~ N(0,1) seeded; image tokens split 2-way by sequence, text
replicated; each rank's result checked against single-process attention.
Also the ring restatement, the all-to-all round trip, and the peer-window
handle exchange of the product's host code.
"""
from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, fn, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.set_num_threads(max(1, (os.cpu_count() or 2) // world))
        fn(rank, world)
        q.put((rank, None))
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def spawn(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    errors = [err for _, err in results if err]
    assert not errors, "\n".join(errors)


def _c1_inputs():
    g = torch.Generator().manual_seed(0)
    img = [torch.randn(1, 1024, 8, 64, generator=g) for _ in range(3)]
    txt = [torch.randn(1, 256, 8, 64, generator=g) for _ in range(3)]
    return img, txt


def _c1_worker(rank, world):
    from oracle.gloo_usp import attention_lse_torch, ulysses_joint_attention

    img, txt = _c1_inputs()
    ls = 1024 // world
    local = [t[:, rank * ls:(rank + 1) * ls] for t in img]
    out_img, out_txt = ulysses_joint_attention(*local, *txt)
    full = [torch.cat((t, i), dim=1) for t, i in zip(txt, img)]
    ref, _ = attention_lse_torch(*full)
    torch.testing.assert_close(out_img, ref[:, 256 + rank * ls:256 + (rank + 1) * ls], atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(out_txt, ref[:, :256], atol=2e-5, rtol=1e-4)


def test_c1_joint_ulysses_world2_matches_single_process():
    spawn(_c1_worker)


def _ring_worker(rank, world):
    from oracle.gloo_usp import attention_lse_torch, ring_attention

    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, 96 * world, 4, 32, generator=g, dtype=torch.float64) for _ in range(3))
    sl = slice(rank * 96, (rank + 1) * 96)
    out, lse = ring_attention(q[:, sl], k[:, sl], v[:, sl])
    ref, ref_lse = attention_lse_torch(q, k, v)
    torch.testing.assert_close(out, ref[:, sl], atol=1e-12, rtol=1e-12)
    torch.testing.assert_close(lse, ref_lse[:, :, sl], atol=1e-12, rtol=1e-12)


def test_ring_restatement_world2_is_exact_in_float64():
    spawn(_ring_worker)


def _a2a_worker(rank, world):
    from oracle import usp
    from oracle.gloo_usp import seq_all_to_all_4d

    g = torch.Generator().manual_seed(2)
    locals_ = [torch.randn(2, 10, 6, 8, generator=g) for _ in range(world)]
    got = seq_all_to_all_4d(locals_[rank], 2, 1)
    want = usp.seq_all_to_all_4d([t.numpy() for t in locals_], 2, 1)[rank]
    assert torch.equal(got, torch.from_numpy(want))
    back = seq_all_to_all_4d(got, 1, 2)
    assert torch.equal(back, locals_[rank])


def test_gloo_all_to_all_matches_the_numpy_oracle():
    spawn(_a2a_worker)


def _handles_worker(rank, world):
    from dgx_monarch_b200.comm import _exchange_handles

    mine = bytes([rank * 16 + i for i in range(64)])
    allh = _exchange_handles(mine, None, torch.device("cpu"))
    assert len(allh) == 64 * world
    for r in range(world):
        assert allh[r * 64:(r + 1) * 64] == bytes([r * 16 + i for i in range(64)])


def test_peer_window_handle_exchange_is_rank_ordered():
    spawn(_handles_worker)


@pytest.mark.parametrize("world,uly,ring", [(8, 2, 4), (8, 4, 2), (8, 8, 1), (8, 1, 8), (4, 2, 2),
                                             (16, 2, 4), (6, 3, 2), (2, 1, 2)])
def test_hybrid_layout_matches_the_oracle(world, uly, ring):
    """The package's Ulysses x ring group layout is the oracle's ulysses-low
    restatement, every group a partition of the world."""
    from dgx_monarch_b200.groups import hybrid_layout
    from oracle.usp import hybrid_groups

    got = hybrid_layout(world, uly, ring)
    assert got == hybrid_groups(world, uly, ring)
    for groups, size in zip(got, (uly, ring)):
        assert sorted(r for g in groups for r in g) == list(range(world))
        assert all(len(g) == size for g in groups)


def test_hybrid_layout_refuses_a_world_it_does_not_tile():
    from dgx_monarch_b200.groups import hybrid_layout

    with pytest.raises(ValueError, match="not a multiple"):
        hybrid_layout(6, 2, 2)


def _groups_worker(rank, world):
    from dgx_monarch_b200.groups import new_hybrid_groups

    for uly, ring in ((2, 1), (1, 2)):
        ug, rg = new_hybrid_groups(world, uly, ring)
        assert dist.get_world_size(ug) == uly and dist.get_world_size(rg) == ring
        # A collective over each group sees exactly that group's ranks.
        for group, size in ((ug, uly), (rg, ring)):
            t = torch.tensor([float(rank + 1)])
            dist.all_reduce(t, group=group)
            assert t.item() == (3.0 if size == 2 else float(rank + 1))


def test_new_hybrid_groups_world2():
    spawn(_groups_worker, 2)
