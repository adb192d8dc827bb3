"""Timed CPU baseline: the reference's attention math on the host cores.

TEST INFRASTRUCTURE ONLY -- the oracle's timing leg, used by bench.py's CPU
baseline and its reference arm.  The reference runs its block attention
through ATen SDPA (adapters/wan_ring_full_context.py:160-167,
adapters/cudnn_ring_attention.py:75-76); on the CPU that is
torch.nn.functional.scaled_dot_product_attention in fp32, which is what is
timed here on a bounded sample of the benchmark's workload: blocks of query
rows of one head at a time against that head's full key/value axis.
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
