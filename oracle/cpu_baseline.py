"""Timed CPU baseline: the reference's attention path on the host cores.

TEST INFRASTRUCTURE ONLY -- the oracle's timing leg, used by bench.py's CPU
baseline and its reference arm, never by the product.

- `time_ulysses_sample`: the reference's pure-Ulysses path
  (adapters/usp_full_axis.py:27-40 at ring world 1) as world-2 gloo
  processes: the all-to-all of q, k and v, fp32 torch SDPA over the whole
  sequence (the reference's ATen SDPA, adapters/wan_ring_full_context.py:
  160-167), the inverse all-to-all -- on a bounded sample of the benchmark's
  heads.
- `time_sdpa_sample`: the inner kernel alone on blocks of query rows.
"""
from __future__ import annotations

import os
import time

import torch


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def time_sdpa_sample(seq_len: int, heads: int, head_dim: int, *, q_rows: int = 1024,
                     budget_s: float = 12.0, threads: int | None = None, seed: int = 0,
                     max_blocks: int | None = None) -> dict:
    """Run fp32 CPU SDPA on (q_rows x seq_len) blocks until `budget_s` elapses.

    Returns achieved TFLOP/s over the warm blocks (the first block is a
    discarded cold run, as the reference's benchmarks discard cold renders).
    """
    threads = threads or host_cores()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(1, 1, seq_len, head_dim, generator=g)
    v = torch.randn(1, 1, seq_len, head_dim, generator=g)
    q = torch.randn(1, 1, q_rows, head_dim, generator=g)
    flops_block = 4.0 * q_rows * seq_len * head_dim
    torch.nn.functional.scaled_dot_product_attention(q, k, v)  # cold run, discarded
    blocks, start = 0, time.perf_counter()
    while True:
        torch.nn.functional.scaled_dot_product_attention(q, k, v)
        blocks += 1
        elapsed = time.perf_counter() - start
        if elapsed >= budget_s or (max_blocks is not None and blocks >= max_blocks):
            break
    tflops = blocks * flops_block / elapsed / 1e12
    return {
        "value": tflops,
        "unit": "TFLOP/s",
        "cores": threads,
        "seconds": elapsed,
        "blocks": blocks,
        "sample": (f"{blocks} blocks of {q_rows} query rows x {seq_len} keys x d{head_dim}, "
                   f"one head each (of {heads}), fp32 torch SDPA on {threads} host threads, "
                   f"{elapsed:.1f} s warm"),
    }


def _ulysses_rank(rank: int, world: int, port: int, seq_len: int, heads: int, head_dim: int,
                  threads: int, steps: int, warmup: int, out_q) -> None:
    """One gloo rank of the timed Ulysses sample (spawned; see time_ulysses_sample)."""
    import torch.distributed as dist

    from oracle.gloo_usp import seq_all_to_all_4d

    try:
        torch.set_num_threads(threads)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        ls = seq_len // world
        g = torch.Generator().manual_seed(1234 + rank)
        q, k, v = (torch.randn(1, ls, heads, head_dim, generator=g) for _ in range(3))
        times = []
        for step in range(warmup + steps):
            dist.barrier()
            start = time.perf_counter()
            qg, kg, vg = (seq_all_to_all_4d(t, 2, 1) for t in (q, k, v))   # (1, S, H/P, D)
            out = torch.nn.functional.scaled_dot_product_attention(
                qg.transpose(1, 2), kg.transpose(1, 2), vg.transpose(1, 2)).transpose(1, 2)
            back = seq_all_to_all_4d(out.contiguous(), 1, 2)                # (1, S/P, H, D)
            elapsed = torch.tensor([time.perf_counter() - start], dtype=torch.float64)
            dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
            if step >= warmup:
                times.append(elapsed.item())
            del qg, kg, vg, out, back
        if rank == 0:
            out_q.put(("ok", times))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # pragma: no cover - reported to the parent
        out_q.put(("error", f"rank {rank}: {type(exc).__name__}: {exc}"))


def time_ulysses_sample(seq_len: int, heads: int, head_dim: int, *, world: int = 2, steps: int = 2,
                        warmup: int = 1, threads: int | None = None) -> dict:
    """The reference's pure-Ulysses data path on the host cores: `world` gloo
    ranks (spawned processes, the host cores split evenly), each holding
    seq_len / world rows of `heads` heads.  One step is the sequence->head
    all-to-all of q, k and v (all_to_all_single in the rank-major order of
    yunchang's SeqAllToAll4D), fp32 torch SDPA over the whole sequence for
    the rank's heads, and the inverse all-to-all (adapters/usp_full_axis.py:
    27-40 at ring world 1).  The step time is the max over ranks; the first
    `warmup` steps are discarded, as the reference's benchmarks discard cold
    renders."""
    import socket

    import torch.multiprocessing as mp

    threads = threads or max(1, host_cores() // world)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    procs = [ctx.Process(target=_ulysses_rank, args=(r, world, port, seq_len, heads, head_dim, threads,
                                                      steps, warmup, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    import queue

    result = None
    while result is None:
        try:
            result = out_q.get(timeout=5)
        except queue.Empty:
            dead = [p for p in procs if not p.is_alive() and p.exitcode not in (0, None)]
            if dead:
                for p in procs:
                    if p.is_alive():
                        p.terminate()
                raise RuntimeError(f"a Ulysses sample rank exited with code {dead[0].exitcode}")
    for p in procs:
        p.join(timeout=120)
    status, payload = result
    if status != "ok":
        raise RuntimeError(payload)
    step_s = sum(payload) / len(payload)
    flops = 4.0 * heads * seq_len * seq_len * head_dim
    return {
        "value": flops / step_s / 1e12,
        "unit": "TFLOP/s",
        "cores": threads * world,
        "step_s": step_s,
        "steps": len(payload),
        "sample": (f"{heads} of the layer's heads over the whole {seq_len}-token axis: world-{world} gloo "
                   f"Ulysses (all-to-all of q/k/v, fp32 torch SDPA, inverse all-to-all), {threads} threads "
                   f"per rank, {step_s:.2f} s per warm step (max over ranks)"),
    }
