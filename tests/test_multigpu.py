"""Ulysses across real GPUs: IPC peer windows, peer stores, flag barriers.

Runs only when at least two CUDA devices are visible; each rank is a child
process on its own GPU (never two ranks on one GPU, so no kernel waits on a
kernel of another launch on the same device).  NCCL carries only the window
handle exchange; NVLS stays off.
"""
from __future__ import annotations

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
    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from datetime import timedelta

        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=60))
        case(rank, world, dev)
        dist.barrier()
        q.put((rank, None))
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))
    finally:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()


def _spawn(case, world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    errors = [e for _, e in results if e]
    assert not errors, "\n".join(errors)


def _ulysses_case(rank, world, dev):
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
    assert (out.float() - ref).abs().max().item() <= BF16_MAX_ABS
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert _lib.device_error() == 0
    uly.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_ulysses_across_gpus_matches_unsharded_attention():
    _spawn(_ulysses_case, min(torch.cuda.device_count(), 4))
