#!/usr/bin/env python
"""Benchmark of the B200 sequence-parallel attention path.

Workload (one "step"): the Wan-style video DiT self-attention layer --
75,600 tokens (1280x720, 81 frames -> 21x90x160 latent, (1,2,2) patches),
40 heads x 128, bf16, non-causal, Q/K/V ~ N(0,1) seeded.  At N GPUs it runs
as Ulysses-N: each rank holds 75,600/N tokens of all 40 heads, the sequence->
head all-to-all hands every rank 40/N heads of the whole sequence, the rank
attends them, and the inverse all-to-all returns its own rows.

Metric: attention TFLOP/s for the whole job (4*B*H*S*S*D per step divided by
the max over ranks of the device time), plus tokens/s of the layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched with torch.distributed.run (one process per GPU).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "attn TFLOP/s + DiT-layer tokens/s at 1/2/4/8 B200; % of roofline"
SEQ, HEADS, DIM, BATCH = 75600, 40, 128, 1
WORKLOAD = ("Wan-style video DiT self-attention: 75,600 tokens (21x90x160 latent, (1,2,2) "
            "patches), 40 heads x 128, bf16, non-causal, Q/K/V ~ N(0,1)")


def attn_flops(b=BATCH, h=HEADS, s=SEQ, d=DIM) -> float:
    return 4.0 * b * h * s * s * d


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--e2e-groups", type=int, default=0,
                   help="head groups the host-streamed e2e step pipelines (must divide the "
                        "40 heads, with a multiple of the GPU count per group); 0: one head per "
                        "GPU per group, 40 / N groups")
    p.add_argument("--p-chunks", type=int, choices=[0, 1, 4], default=0,
                   help="release each block's probabilities to the tensor core in this many "
                        "chunks (0: the library default, 4; 1: the single release)")
    p.add_argument("--one-cta", action="store_true",
                   help="run 16-bit attention on single CTAs instead of CTA pairs (the library "
                        "default), as a cross-check")
    p.add_argument("--profile-case", choices=["attn", "fp8", "f16", "kernels", "nvlink"], default=None,
                   help="instead of the bench: a few launches of one kernel family, sized for a "
                        "profiler capture (attn / fp8 / f16: three attention launches of --case-seq "
                        "tokens x --case-heads heads on one GPU; kernels: every support kernel at the "
                        "Flux/Krea2 block shapes on one GPU; nvlink: rank 0's Ulysses scatter at the "
                        "Wan layer's P = 2 shapes from one process over two GPUs, its peer half "
                        "stored over NVLink)")
    p.add_argument("--case-seq", type=int, default=32768)
    p.add_argument("--case-heads", type=int, default=8)
    p.add_argument("--case-batch", type=int, default=1)
    return p.parse_args()


# ----------------------------------------------------------------- profiler cases
def run_profile_case(args) -> None:
    """Representative launches for an ncu capture: small enough (a few GB on
    the device, inputs above the 126 MB L2) that a full-set capture of one
    launch ends in a minute or two."""
    import torch

    from dgx_monarch_b200.ops import attention_fwd, set_p_chunks

    set_p_chunks(args.p_chunks)
    if args.one_cta:
        from dgx_monarch_b200.ops import set_cta_pair

        set_cta_pair(False)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    shape = (args.case_batch, args.case_seq, args.case_heads, DIM)
    if args.profile_case == "kernels":
        profile_support_kernels(dev, g)
        return
    if args.profile_case == "nvlink":
        profile_nvlink_scatter(g)
        return
    if args.profile_case == "fp8":
        from dgx_monarch_b200.prologue import quantize_e4m3_per_head

        q8, k8, v8 = (quantize_e4m3_per_head(torch.randn(*shape, device=dev, generator=g).bfloat16())
                      for _ in range(3))
        out = torch.empty(*shape, device=dev, dtype=torch.bfloat16)
        for _ in range(3):
            attention_fwd(q8[0], k8[0], v8[0], q_descale=q8[1], k_descale=k8[1], v_descale=v8[1],
                          out=out, return_lse=False)
    else:
        dt = torch.float16 if args.profile_case == "f16" else torch.bfloat16
        q, k, v = (torch.randn(*shape, device=dev, generator=g).to(dt) for _ in range(3))
        out = torch.empty_like(q)
        for _ in range(3):
            attention_fwd(q, k, v, out=out, return_lse=False)
    torch.cuda.synchronize()


def profile_nvlink_scatter(g) -> None:
    """Rank 0's sequence->head scatter of the Wan layer at P = 2, in one process
    over two GPUs: q/k/v (37,800 local rows x 40 heads x 128, bf16) on cuda:0,
    head slice [0, 20) stored into rank 0's receive tensors on cuda:0 and head
    slice [20, 40) into rank 1's on cuda:1 through peer access -- 580.6 MB over
    NVLink per launch; then the store half of the ring-2 full-context K/V
    gather, rank 0's K and V into both ranks' full K/V -- 774.1 MB over NVLink
    per launch.  For the launching GPU's NVLink byte counters; three launches
    of each, the last timed with CUDA events."""
    import torch
    from cuda.bindings import runtime as cudart

    from dgx_monarch_b200.ulysses import ulysses_scatter

    if torch.cuda.device_count() < 2:
        raise SystemExit("the nvlink case needs two GPUs in this process")
    torch.cuda.set_device(0)
    (err,) = cudart.cudaDeviceEnablePeerAccess(1, 0)
    if err not in (cudart.cudaError_t.cudaSuccess, cudart.cudaError_t.cudaErrorPeerAccessAlreadyEnabled):
        raise SystemExit(f"peer access from GPU 0 to GPU 1: {err}")
    ls, h = SEQ // 2, HEADS
    x = [torch.randn(1, ls, h, DIM, device="cuda:0", generator=g).bfloat16() for _ in range(3)]
    recv = [[torch.empty(1, 2 * ls, h // 2, DIM, device=f"cuda:{r}", dtype=torch.bfloat16) for r in range(2)]
            for _ in range(3)]
    dst = [[recv[t][r].data_ptr() for r in range(2)] for t in range(3)]
    for _ in range(2):
        ulysses_scatter(x, dst, world=2, rank=0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    ulysses_scatter(x, dst, world=2, rank=0)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    peer_bytes = 3 * ls * (h // 2) * DIM * 2
    print(f"scatter {ms:.3f} ms, {peer_bytes / 1e6:.1f} MB to the peer: {peer_bytes / ms / 1e6:.1f} GB/s per direction")
    # The peer half arrived: rank 1's receive rows [0, ls) hold heads [20, 40).
    assert torch.equal(recv[0][1][0, :ls].to("cuda:0"), x[0][0, :, h // 2:])
    del recv
    # The store half of the Wan ring-2 full-context gather: rank 0's K/V block
    # (37,800 rows x 40 heads x 128) into rows [0, ls) of both ranks' full K/V.
    from dgx_monarch_b200.ring import kv_gather_store

    k, v = x[1], x[2]
    full = [[torch.empty(1, 2 * ls, h, DIM, device=f"cuda:{r}", dtype=torch.bfloat16) for r in range(2)]
            for _ in range(2)]
    dk, dv = [t.data_ptr() for t in full[0]], [t.data_ptr() for t in full[1]]
    for _ in range(2):
        kv_gather_store(k, v, dk, dv, world=2, rank=0)
    e0.record()
    kv_gather_store(k, v, dk, dv, world=2, rank=0)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    peer_bytes = 2 * ls * h * DIM * 2
    print(f"kv gather store {ms:.3f} ms, {peer_bytes / 1e6:.1f} MB to the peer: "
          f"{peer_bytes / ms / 1e6:.1f} GB/s per direction")
    assert torch.equal(full[1][1][0, :ls].to("cuda:0"), v[0])


def profile_support_kernels(dev, g) -> None:
    """Every support kernel once or twice, at the C2 (Flux/Krea2 block) and C3
    shapes on one rank, each input larger than the L2 where the kernel is
    HBM-bound."""
    import torch

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.cfg import cfg_combine
    from dgx_monarch_b200.ops import lse_merge
    from dgx_monarch_b200.prologue import (qkv_gemm_prologue_scatter, qkv_prologue_scatter,
                                           quantize_e4m3_per_head, rope_table)
    from dgx_monarch_b200.shard import SequenceGather, SharedActivationScale
    from dgx_monarch_b200.ulysses import ulysses_scatter_joint

    hid, heads, rows = 3072, 24, 9728
    w = lambda *s, sc=0.02: (sc * torch.randn(*s, device=dev, generator=g)).bfloat16()
    x = w(rows, hid, sc=1.0)
    wq, bq = w(3 * hid, hid), w(3 * hid)
    nq, nk = (1 + w(128)).contiguous(), (1 + w(128)).contiguous()
    pos = torch.stack((torch.zeros(rows, device=dev, dtype=torch.long),
                       torch.arange(rows, device=dev) // 96, torch.arange(rows, device=dev) % 96), dim=1)
    table = rope_table(pos, [16, 56, 56])
    recv = [torch.empty(rows, heads, 128, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    dst = [[t.data_ptr()] for t in recv]
    for _ in range(2):
        qkv_gemm_prologue_scatter(x, wq, dst, world=1, rank=0, seq_local=rows, bias=bq,
                                  norm_mode=_lib.NORM_HEAD, norm_q_w=nq, norm_k_w=nk, rope=table)
    qkv = (x @ wq.t()).view(1, rows, 3, heads, 128)
    for _ in range(2):
        qkv_prologue_scatter(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], dst, world=1, rank=0,
                             norm_mode=_lib.NORM_HEAD, norm_q_w=nq, norm_k_w=nk, rope=table)
    del qkv
    txt_rows = 512
    joint = [torch.empty(1, rows, heads, 128, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    img = [w(1, rows - txt_rows, heads, 128, sc=1.0) for _ in range(3)]
    txt = [w(1, txt_rows, heads, 128, sc=1.0) for _ in range(3)]
    for _ in range(2):
        ulysses_scatter_joint(img, txt, [[t.data_ptr()] for t in joint], world=1, rank=0)
    del joint, img, txt
    xq = torch.randn(1, 32768, 24, 128, device=dev, generator=g).bfloat16()
    for _ in range(2):
        quantize_e4m3_per_head(xq)
    parts = [torch.randn(1, 32768, 8, 128, device=dev, generator=g) for _ in range(2)]
    lses = [torch.randn(1, 8, 32768, device=dev, generator=g) for _ in range(2)]
    for _ in range(2):
        lse_merge(parts, lses)
    c, u = (torch.randn(64 * 1024 * 1024, device=dev, generator=g) for _ in range(2))
    for _ in range(2):
        cfg_combine(c, u, 4.0)
    del c, u
    act = w(rows, 3 * hid, sc=1.0)
    scale = SharedActivationScale(device=dev, generation=90)
    for _ in range(2):
        scale(act)
    scale.close()
    gather = SequenceGather(device=dev, generation=91)
    tokens = w(2, rows, hid, sc=1.0)
    for _ in range(2):
        gather(tokens, rows)
    gather.close()
    torch.cuda.synchronize()


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of this GPU's clocks during the timed region."""

    FIELDS = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str) -> None:
        self.bus_id = bus_id.lower()
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def wait_first(self, timeout_s: float = 10.0) -> None:
        """Block until the first sample has arrived (nvidia-smi can take a
        second to start when every rank launches one), so that the timed
        region that follows is sampled."""
        deadline = time.monotonic() + timeout_s
        while self.proc is not None and not self.rows and time.monotonic() < deadline:
            time.sleep(0.02)

    def _read(self) -> None:
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9 and parts[0].lower().endswith(self.bus_id[-12:]):
                self.rows.append(parts)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        loaded = [s for s in sm if s > 0.5 * (max(mx) if mx else 1)] or sm
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def bus_id_of(device_index: int) -> str:
    import torch

    p = torch.cuda.get_device_properties(device_index)
    return f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"


# ----------------------------------------------------------------- peaks / traffic
def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "bf16_sustained": d["bf16_tflops_sustained"],
                "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def profiled_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    table = json.loads(path.read_text())
    entry = table.get(f"{kernel}:{workload}")
    return None if entry is None else entry.get("bytes_per_launch")


# ----------------------------------------------------------------- reference arm
REF_SAMPLE_HEADS = 2  # heads of the layer the CPU reference path attends per step


def run_reference(args) -> None:
    """The reference's own path on the host cores: pure Ulysses at world 2 over
    gloo (the all-to-all of q/k/v, fp32 torch SDPA, the inverse all-to-all),
    each step a sample of the layer -- 2 of its 40 heads over the whole
    75,600-token axis -- timed as the max over the two ranks.  Under torchrun
    rank 0 alone runs it; the metric is the layer's attention TFLOP/s."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.cpu_baseline import time_ulysses_sample

    r = time_ulysses_sample(SEQ, REF_SAMPLE_HEADS, DIM, world=2, steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": r["value"], "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["step_s"] * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (Q/K/V ~ N(0,1), seeded)",
        "config": {"workload": WORKLOAD, "seq_len": SEQ, "heads": HEADS, "head_dim": DIM,
                   "batch": BATCH, "parallelism": "ulysses2 over gloo on the host cores",
                   "step": f"{REF_SAMPLE_HEADS} of the {HEADS} heads over the whole axis per step"},
        "cpu_baseline": {"value": r["value"], "unit": "TFLOP/s", "cores": r["cores"], "kind": "port",
                         "sample": r["sample"]},
        "e2e": {"value": r["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- DiT layer
DIT = {"hidden": 3072, "heads": 24, "img": 9216, "txt": 512, "latent": (96, 96)}
DIT_WORKLOAD = ("Flux/Krea2-style joint-attention DiT double block (attention sub-layer): "
                "1536x1536 image -> 96x96 patch grid = 9216 tokens + 512 text tokens, hidden 3072, "
                "24 heads x 128, bf16, random-init weights N(0, 0.02); QKV projection with bias, "
                "per-head RMSNorm on Q/K, 2-axis RoPE and the sequence->head scatter (one fused tcgen05 "
                "GEMM launch for both streams, or cuBLAS + the prologue kernel, whichever this run timed faster: "
                "qkv_stage_ms.in_layer), joint [text, image] attention with the inverse all-to-all in its "
                "epilogue, out projection (cuBLAS)")


def time_steps(step, steps: int, warmup: int, graph: bool = False) -> float:
    """Mean device ms per step over `steps` timed steps, eagerly or as a
    replayed CUDA graph of one step (captured after the warm-up; every rank
    captures and replays the same sequence)."""
    import torch

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    run, captured = step, None
    if graph:
        captured = torch.cuda.CUDAGraph()
        with torch.cuda.graph(captured):
            step()
        run = captured.replay
        for _ in range(warmup):
            run()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    del captured
    return e0.elapsed_time(e1) / steps


def check_sampled_rows(out, world: int, rank: int, dev, ls: int, n_rows: int = 64) -> dict:
    """The timed step's output on a sample of this rank's query rows (all
    heads) against fp32 attention over the whole key axis, outside the timed
    region.  Every rank's seeded inputs are regenerated here (same seeds, same
    generator), so each rank checks its own rows against every key.  Bounds:
    bf16 max-abs 2e-2, rel-L2 5e-3; the result is the max over ranks."""
    import torch
    import torch.distributed as dist

    ks, vs, q_local = [], [], None
    for r in range(world):
        g = torch.Generator(device=dev).manual_seed(1234 + r)
        q_r, k_r, v_r = (torch.randn(BATCH, ls, HEADS, DIM, device=dev, generator=g, dtype=torch.bfloat16)
                         for _ in range(3))
        ks.append(k_r)
        vs.append(v_r)
        if r == rank:
            q_local = q_r
    k, v = torch.cat(ks, dim=1).float(), torch.cat(vs, dim=1).float()
    del ks, vs
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    rows = torch.cat((torch.randint(0, ls, (n_rows - 8,), device=dev, generator=g),
                      torch.arange(ls - 8, ls, device=dev)))
    qs = q_local[:, rows].float().permute(0, 2, 1, 3)                    # B H n D
    logits = torch.matmul(qs, k.permute(0, 2, 3, 1)) / math.sqrt(DIM)    # B H n S
    ref = torch.matmul(torch.softmax(logits, dim=-1), v.permute(0, 2, 1, 3)).permute(0, 2, 1, 3)
    got = out[:, rows].float()
    err = torch.tensor([(got - ref).abs().max().item(),
                        ((got - ref).norm() / ref.norm()).item()], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
    max_abs, rel = err.tolist()
    return {"rows_per_rank": n_rows, "heads": HEADS, "against": "fp32 attention over all keys",
            "max_abs": max_abs, "rel_l2": rel, "ok": bool(max_abs <= 2e-2 and rel <= 5e-3)}


def dit_layer_flops() -> float:
    s, hid = DIT["img"] + DIT["txt"], DIT["hidden"]
    return 2.0 * s * hid * 3 * hid + 2.0 * s * hid * hid + attn_flops(1, DIT["heads"], s, DIM)


def run_dit_layer(world: int, rank: int, dev, steps: int, warmup: int, group=None) -> dict:
    """One C2 double-block attention sub-layer per step, Ulysses over `world`."""
    import torch

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.comm import PeerWindows
    from dgx_monarch_b200.prologue import qkv_gemm_prologue_scatter_streams, qkv_prologue_scatter, rope_table
    from dgx_monarch_b200.ulysses import attention_routed

    hid, h = DIT["hidden"], DIT["heads"]
    t_loc, i_loc = DIT["txt"] // world, DIT["img"] // world
    ls = t_loc + i_loc
    s = ls * world
    hl = h // world
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    w = lambda *shape: (0.02 * torch.randn(*shape, device=dev, generator=g)).bfloat16()
    x_txt, x_img = w(1, t_loc, hid) * 50, w(1, i_loc, hid) * 50
    # Linear weights (out, in), as the block's modules hold them, and their biases.
    w_qkv_txt, w_qkv_img = w(3 * hid, hid), w(3 * hid, hid)
    b_qkv_txt, b_qkv_img = w(3 * hid), w(3 * hid)
    qkv = torch.empty(1, ls, 3, h, DIM, device=dev, dtype=torch.bfloat16)
    w_o_txt, w_o_img = w(hid, hid), w(hid, hid)
    nq, nk = (1 + w(128)).contiguous(), (1 + w(128)).contiguous()
    # Positions: text tokens at 0, image tokens at (0, row, col) of the 96x96 grid.
    img_ids = torch.arange(rank * i_loc, (rank + 1) * i_loc, device=dev)
    pos = torch.cat((torch.zeros(t_loc, 3, device=dev, dtype=torch.long),
                     torch.stack((torch.zeros_like(img_ids), img_ids // 96, img_ids % 96), dim=1)))
    table = rope_table(pos, [16, 56, 56])
    elt = 2
    recv_bytes = s * hl * DIM * elt
    out_bytes = ls * h * DIM * elt
    win = PeerWindows(3 * recv_bytes + out_bytes + 1024, device=dev, group=group, rank=rank,
                      world=world, generation=11)
    offs = [win.carve(recv_bytes) for _ in range(3)] + [win.carve(out_bytes)]
    recv = [win.local_tensor(o, (1, s, hl, DIM), torch.bfloat16) for o in offs[:3]]
    out_local = win.local_tensor(offs[3], (1, ls, h, DIM), torch.bfloat16)
    y = torch.empty(1, ls, hid, device=dev, dtype=torch.bfloat16)

    dst = [[win.peer_ptr(r, o) for r in range(world)] for o in offs[:3]]

    def qkv_fused():
        # QKV Linear + QKNorm + RoPE + sequence->head scatter of both streams, one launch.
        qkv_gemm_prologue_scatter_streams(
            [dict(x=x_txt, w_qkv=w_qkv_txt, bias=b_qkv_txt, norm_q_w=nq, norm_k_w=nk, row0=0),
             dict(x=x_img, w_qkv=w_qkv_img, bias=b_qkv_img, norm_q_w=nq, norm_k_w=nk, row0=t_loc)],
            dst, world=world, rank=rank, seq_local=ls, seg0=t_loc, norm_mode=_lib.NORM_HEAD, rope=table)

    def qkv_split():
        # cuBLAS QKV Linear per stream, then the fused norm + RoPE + scatter kernel.
        torch.addmm(b_qkv_txt, x_txt[0], w_qkv_txt.t(), out=qkv[0, :t_loc].view(t_loc, 3 * hid))
        torch.addmm(b_qkv_img, x_img[0], w_qkv_img.t(), out=qkv[0, t_loc:].view(i_loc, 3 * hid))
        qkv_prologue_scatter(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], dst, world=world, rank=rank,
                             norm_mode=_lib.NORM_HEAD, norm_q_w=nq, norm_k_w=nk, rope=table, seg0=t_loc)

    # The QKV stage alone, both ways (rank-local work; peers are not waited for).
    # The layer runs the faster one, the same on every rank (max over ranks): the
    # fused GEMM wins at 1-4 ranks, cuBLAS + the prologue kernel at 8, where a
    # rank projects only 1216 rows.
    ms_split = time_steps(qkv_split, steps, warmup, graph=True)
    ms_fused = time_steps(qkv_fused, steps, warmup, graph=True)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms_split, ms_fused], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        ms_split, ms_fused = t.tolist()
    qkv_stage = qkv_fused if ms_fused <= ms_split else qkv_split

    def step():
        qkv_stage()
        win.barrier()
        attention_routed(recv[0], recv[1], recv[2], [win.peer_ptr(r, offs[3]) for r in range(world)],
                         (ls * h * DIM, h * DIM, DIM), world=world, rank=rank, seq_local=ls, seg0=t_loc)
        win.barrier()
        o = out_local.view(1, ls, hid)
        torch.matmul(o[:, :t_loc], w_o_txt, out=y[:, :t_loc])
        torch.matmul(o[:, t_loc:], w_o_img, out=y[:, t_loc:])

    ms_eager = time_steps(step, steps, warmup)
    ms = time_steps(step, steps, warmup, graph=True)  # the same work, launched from one graph
    if world > 1:
        win.barrier()
        torch.cuda.synchronize()
    win.close()
    fused = qkv_stage is qkv_fused
    return {"ms": ms, "ms_eager": ms_eager, "ms_qkv_split": ms_split, "ms_qkv_fused": ms_fused,
            "qkv_fused_in_layer": fused,
            "my_launches": 6 if world > 1 else 4}


# ----------------------------------------------------------------- ring / CFG workloads (N > 1)
RING = {"seq": 219600, "heads": 24}
RING_WORKLOAD = ("Long-video hybrid ring x Ulysses attention: 1280x720 at 241 frames -> 61x90x160 "
                 "latent, (1,2,2) patches = 219,600 tokens, 24 heads x 128, bf16; Ulysses-2 x ring-N/2 "
                 "(ring-2 at N=2), K/V blocks rotating over NVLink, LSE merge")
CFG = {"img": 4096, "txt": 512, "heads": 24, "batch": 2}
CFG_WORKLOAD = ("CFG-parallel + Ulysses image attention: batch 2 (cond/uncond) -> one row per cfg rank, "
                "1024x1024 image = 4096 tokens + 512 text tokens, 24 heads x 128, Q/K/V in FP8 e4m3 with "
                "per-head absmax scales, bf16 out; cfg2 x Ulysses-N/2")


def _groups(world: int, uly: int, ring: int):
    """This rank's Ulysses / ring process groups in the ulysses-low layout
    (Ulysses groups are consecutive ranks), every rank creating every group."""
    from dgx_monarch_b200.groups import new_hybrid_groups

    return new_hybrid_groups(world, uly, ring)


def run_ring(world: int, rank: int, dev, steps: int, warmup: int) -> dict:
    import torch

    from dgx_monarch_b200.usp import make_b200_usp_attention

    uly = 2 if world >= 4 else 1
    ring = world // uly
    ug, rg = _groups(world, uly, ring)
    attn = make_b200_usp_attention(ulysses_group=ug if uly > 1 else None, ring_group=rg,
                                   generation=31, device=dev)
    seq, h = RING["seq"], RING["heads"]
    ls = seq // world
    g = torch.Generator(device=dev).manual_seed(500 + rank)
    q, k, v = (torch.randn(1, ls, h * DIM, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(3))
    for _ in range(warmup):
        attn(q, k, v, heads=h)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        attn(q, k, v, heads=h)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    attn.impl.invalidate()
    return {"ms": ms, "layout": f"ulysses{uly}xring{ring}"}


def run_full_context(world: int, rank: int, dev, steps: int, warmup: int) -> dict:
    """The Wan Ring2 full-context path on the C4 layer: ranks in pairs, each
    pair a pure ring of degree 2 gathering K/V over NVLink and attending
    local Q against the full 75,600-key axis in one call."""
    import torch
    import torch.distributed as dist

    from dgx_monarch_b200.usp import make_b200_usp_attention

    mine = None
    for first in range(0, world - world % 2, 2):
        g = dist.new_group([first, first + 1])
        if rank in (first, first + 1):
            mine = g
    attn = make_b200_usp_attention(ring_group=mine, generation=33, device=dev, full_context_ring=True)
    ls = SEQ // 2
    g = torch.Generator(device=dev).manual_seed(700 + rank)
    q, k, v = (torch.randn(1, ls, HEADS * DIM, device=dev, generator=g, dtype=torch.bfloat16)
               for _ in range(3))
    for _ in range(warmup):
        attn(q, k, v, heads=HEADS)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        attn(q, k, v, heads=HEADS)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    attn.impl.invalidate()
    return {"ms": ms, "pairs": world // 2}


def run_cfg_fp8(world: int, rank: int, dev, steps: int, warmup: int) -> dict:
    """C3: the cond/uncond pair in e4m3.  At N > 1 the pair maps to GPU pairs
    (cfg2 x Ulysses-N/2: each cfg rank attends its batch row's sequence shard,
    then the predictions are all-gathered over the pair); at N = 1 one call
    attends both rows.  Also measures the output against fp32 attention of the
    e4m3 inputs and of the bf16 activations (max over ranks)."""
    import torch
    import torch.distributed as dist

    from dgx_monarch_b200.cfg import CfgGather
    from dgx_monarch_b200.usp import make_b200_usp_attention

    s, h = CFG["img"] + CFG["txt"], CFG["heads"]
    if world == 1:
        sp, rows, seeds = 1, 2, [700, 701]
        attn = make_b200_usp_attention(generation=41, device=dev, fp8=True)
        gather = None
    else:
        sp = world // 2
        # sequence parallel fastest, then cfg: ranks r and r + sp form a cond/uncond pair
        mine_sp = mine_cfg = None
        for ranks in [list(range(c * sp, (c + 1) * sp)) for c in range(2)]:
            gsp = dist.new_group(ranks)
            if rank in ranks:
                mine_sp = gsp
        for ranks in [[r, r + sp] for r in range(sp)]:
            gc = dist.new_group(ranks)
            if rank in ranks:
                mine_cfg = gc
        attn = make_b200_usp_attention(ulysses_group=mine_sp if sp > 1 else None, generation=41,
                                       device=dev, fp8=True)
        rows, seeds = 1, [700 + rank]
    ls = s // sp

    def inputs(seed_list):
        qkv = []
        for seed in seed_list:
            g = torch.Generator(device=dev).manual_seed(seed)
            qkv.append([torch.randn(1, ls, h * DIM, device=dev, generator=g, dtype=torch.bfloat16)
                        for _ in range(3)])
        return [torch.cat([x[t] for x in qkv]) for t in range(3)]

    q, k, v = inputs(seeds)
    if world > 1:
        gather = CfgGather(ls * h * DIM * 2, device=dev, group=mine_cfg, generation=41)

    def step():
        out = attn(q, k, v, heads=h)          # this cfg rank's batch row(s), its sequence shard
        return out if gather is None else gather(out)

    ms_eager = time_steps(step, steps, warmup)
    ms = time_steps(step, steps, warmup, graph=world > 1)
    out = attn(q, k, v, heads=h).float().view(rows, ls, h, DIM)
    # This rank's rows against fp32 attention over its batch row's whole
    # sequence, rebuilt from the seeds of the ranks holding that row.
    row_seeds = seeds if world == 1 else [700 + (rank // sp) * sp + r for r in range(sp)]
    full = [x.view(-1, s if world == 1 else ls, h, DIM) for x in inputs(row_seeds)]
    if world > 1:
        full = [x.reshape(1, s, h, DIM) for x in full]
    mine = slice(0, s) if world == 1 else slice((rank % sp) * ls, (rank % sp + 1) * ls)

    def attend(qf, kf, vf):
        logits = torch.einsum("bqhd,bkhd->bhqk", qf, kf) / math.sqrt(DIM)
        return torch.einsum("bhqk,bkhd->bqhd", torch.softmax(logits, dim=-1), vf)

    def e4m3(x):
        scale = x.float().abs().amax(dim=(0, 1, 3)).clamp_min(1e-12) / 448.0
        return (x.float() / scale.view(1, 1, -1, 1)).to(torch.float8_e4m3fn).float() * scale.view(1, 1, -1, 1)

    ref_act = attend(*(x.float() for x in full))[:, mine]
    ref_deq = attend(*(e4m3(x) for x in full))[:, mine]
    rel = lambda a, b: ((a - b).norm() / b.norm()).item()
    acc = torch.tensor([rel(out, ref_deq), rel(out, ref_act), rel(ref_deq, ref_act)], device=dev,
                       dtype=torch.float64)
    if world > 1:
        dist.all_reduce(acc, op=dist.ReduceOp.MAX)
        gather.close()
    attn.impl.invalidate()
    vs_inputs, vs_act, floor = acc.tolist()
    return {"ms": ms, "ms_eager": ms_eager, "layout": f"cfg2xulysses{sp}" if world > 1 else "one GPU, both rows",
            "accuracy": {"rel_l2_vs_sdpa_of_e4m3_inputs": vs_inputs, "bound": 3e-2,
                         "rel_l2_vs_sdpa_of_bf16_activations": vs_act,
                         "e4m3_input_floor_vs_activations": floor,
                         "note": "the configuration's attention inputs are the e4m3 tensors; against the "
                                 "unquantized activations the three e4m3 roundings alone give the floor"}}


def time_scatter(uly, steps: int = 5) -> dict:
    """Device time of the Ulysses scatter alone (q, k, v peer stores)."""
    import torch

    from dgx_monarch_b200.ulysses import ulysses_scatter

    w = uly.windows
    q = torch.zeros(uly.b, uly.ls, uly.h, uly.d, device=uly.device, dtype=uly.dtype)
    ptrs = [[w.peer_ptr(r, off) for r in range(uly.world)] for off in uly.off_recv]
    ulysses_scatter([q, q, q], ptrs, world=uly.world, rank=uly.rank)
    w.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        ulysses_scatter([q, q, q], ptrs, world=uly.world, rank=uly.rank)
    e1.record()
    torch.cuda.synchronize()
    w.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    remote = 3 * q.numel() * q.element_size() * (uly.world - 1) / uly.world
    return {"ms": ms, "nvlink_bytes_per_rank": remote, "gbs_per_direction": remote / (ms * 1e-3) / 1e9}


# ----------------------------------------------------------------- our arm
def main() -> None:
    args = parse_args()
    if args.profile_case is not None:
        run_profile_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if args.e2e_groups == 0 and args.gpus >= 1 and HEADS % args.gpus == 0:
        args.e2e_groups = HEADS // args.gpus
    if args.e2e_groups < 1 or HEADS % args.e2e_groups or (HEADS // args.e2e_groups) % args.gpus:
        raise SystemExit(f"--e2e-groups {args.e2e_groups}: groups must divide the {HEADS} heads into "
                         f"groups whose size is a multiple of {args.gpus} GPUs")
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if args.p_chunks:
        from dgx_monarch_b200.ops import set_p_chunks

        set_p_chunks(args.p_chunks)
    if args.one_cta:
        from dgx_monarch_b200.ops import set_cta_pair

        set_cta_pair(False)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.ulysses import OverlappedUlysses, UlyssesAttention

    if SEQ % world or HEADS % world:
        raise SystemExit(f"{world} GPUs do not tile {SEQ} tokens x {HEADS} heads")
    ls = SEQ // world
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    q, k, v = (torch.randn(BATCH, ls, HEADS, DIM, device=dev, generator=g, dtype=torch.bfloat16)
               for _ in range(3))
    uly = UlyssesAttention(world=world, rank=rank, batch=BATCH, seq_local=ls, heads=HEADS,
                           head_dim=DIM, device=dev)
    out = torch.empty(BATCH, ls, HEADS, DIM, device=dev, dtype=torch.bfloat16)
    # N > 1: a first group of one head per rank, whose attention hides the
    # scatter of the other heads (the inverse all-to-all is in the epilogue).
    over_groups = [world, HEADS - world]
    over = (OverlappedUlysses(world=world, rank=rank, batch=BATCH, seq_local=ls, heads=HEADS, head_dim=DIM,
                              device=dev, groups=over_groups, generation=13) if world > 1 else None)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, n):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            fn(q, k, v, out=out)
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    for _ in range(args.warmup):
        uly.forward(q, k, v, out=out)
        if over is not None:
            over.forward(q, k, v, out=out)
    # N > 1: both schedules of the step, two steps each; every rank takes the
    # max over ranks, so all pick the same one for the timed region.
    plain_ms = over_ms = None
    runner = uly
    if over is not None:
        pick = torch.tensor([timed(uly.forward, 2), timed(over.forward, 2)], device=dev, dtype=torch.float64)
        dist.all_reduce(pick, op=dist.ReduceOp.MAX)
        plain_ms, over_ms = pick.tolist()
        runner = over if over_ms < plain_ms else uly

    def step():
        runner.forward(q, k, v, out=out)

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(bus_id_of(local_rank))
    clocks.start()
    clocks.wait_first()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms_local = e0.elapsed_time(e1) / args.steps
    # The attention kernel alone, timed on its own stream (roofline numerator).
    attn_ms_local = uly.time_attention_kernel(args.steps)
    t = torch.tensor([ms_local, attn_ms_local], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, attn_ms = t.tolist()
    launches = args.steps * runner.launches_per_step
    check = check_sampled_rows(out, world, rank, dev, ls)

    # End to end through the public call with host buffers: pinned host Q/K/V in,
    # output back to pinned host memory, every step.
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    hout = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)

    # Groups of heads (5 x 8 by default), each its own Ulysses step: the PCIe
    # copies of group g +/- 1 overlap the all-to-all and attention of group g
    # (ulysses.HostStreamedUlysses).
    from dgx_monarch_b200.ulysses import HostStreamedUlysses

    streamed = HostStreamedUlysses(world=world, rank=rank, batch=BATCH, seq_local=SEQ // world, heads=HEADS,
                                   head_dim=DIM, device=dev, groups=args.e2e_groups, generation=12)

    def e2e_step():
        streamed(hq, hk, hv, hout)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    e2e_steps = max(2, args.steps // 2)
    for _ in range(e2e_steps):
        e2e_step()
    f1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([f0.elapsed_time(f1) / e2e_steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = te.item()
    dit = run_dit_layer(world, rank, dev, max(5, args.steps), args.warmup)
    extra = [dit["ms"], 0.0, 0.0, 0.0, 0.0, 0.0, dit["ms_eager"], 0.0, dit["ms_qkv_split"], dit["ms_qkv_fused"]]
    a2a = ring_res = cfg_res = fc_res = None
    cfg_res = run_cfg_fp8(world, rank, dev, 5, 3)
    extra[3], extra[7] = cfg_res["ms"], cfg_res["ms_eager"]
    if world > 1:
        a2a = time_scatter(uly)
        ring_res = run_ring(world, rank, dev, 2, 1)
        fc_res = run_full_context(world, rank, dev, 3, 3)
        extra[1], extra[2], extra[4], extra[5] = a2a["ms"], ring_res["ms"], a2a["gbs_per_direction"], fc_res["ms"]
    td = torch.tensor(extra, device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(td, op=dist.ReduceOp.MAX)
        # the slowest rank's link rate
        tmin = torch.tensor([extra[4]], device=dev, dtype=torch.float64)
        dist.all_reduce(tmin, op=dist.ReduceOp.MIN)
        td[4] = tmin[0]
    dit_ms, a2a_ms, ring_ms, cfg_ms, a2a_gbs, fc_ms, dit_ms_eager, cfg_ms_eager, qkv_split_ms, qkv_fused_ms = td.tolist()
    dev_err = _lib.device_error()

    if rank == 0:
        peaks = measured_peaks()
        flops = attn_flops()
        value = flops / (ms * 1e-3) / 1e12
        per_rank_flops = flops / world
        achieved = per_rank_flops / (attn_ms * 1e-3) / 1e12
        pair = not args.one_cta and args.p_chunks != 1
        traffic = profiled_traffic("attn_fwd_bf16_pair" if pair else "attn_fwd_bf16", f"s{SEQ}_h{HEADS // world}")
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak" if world == 1 else "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (Q/K/V ~ N(0,1), seeded)",
            "config": {"workload": WORKLOAD, "seq_len": SEQ, "heads": HEADS, "head_dim": DIM,
                       "batch": BATCH, "parallelism": f"ulysses{world}",
                       "l2": "inputs larger than L2 (Q/K/V 2.3 GB)",
                       "p_chunks": args.p_chunks or "library default (4)"},
            "tokens_per_s": BATCH * SEQ / (ms * 1e-3),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                         "traffic": traffic, "peak_source": peaks["source"] + " burst bf16",
                         "kernel": "attn_fwd_kernel<bf16>" + (" on CTA pairs" if pair else " on single CTAs")},
            "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": 3 * q.numel() * q.element_size(),
                    "d2h_bytes_per_step": out.numel() * out.element_size(),
                    "ms_per_step": e2e_ms,
                    "method": (f"pinned host Q/K/V in, pinned host output back, every step; {args.e2e_groups} "
                               f"groups of {HEADS // args.e2e_groups} heads streamed so the PCIe copies of one "
                               "group overlap the Ulysses step of another (HostStreamedUlysses)")},
            "dit_layer": {"workload": DIT_WORKLOAD, "tokens_per_s": (DIT["img"] + DIT["txt"]) / (dit_ms * 1e-3),
                          "ms_per_layer": dit_ms, "ms_per_layer_eager": dit_ms_eager,
                          "launch": "one CUDA graph per layer (ms_per_layer_eager: the same calls from Python)",
                          "qkv_stage_ms": {"cublas_addmm_plus_prologue_scatter": qkv_split_ms,
                                           "fused_tcgen05_gemm_prologue_scatter": qkv_fused_ms,
                                           "in_layer": ("fused_tcgen05_gemm_prologue_scatter" if qkv_fused_ms <= qkv_split_ms
                                                        else "cublas_addmm_plus_prologue_scatter")},
                          "tflops": dit_layer_flops() / (dit_ms * 1e-3) / 1e12,
                          "frac_of_bf16_peak": dit_layer_flops() / (dit_ms * 1e-3) / 1e12 / (world * peaks["bf16_tflops"]),
                          "parallelism": f"ulysses{world}"},
            "gpu_launches": launches,
            "ulysses_step": ({"timed_schedule": "overlapped" if runner is over else "plain",
                              "overlapped_ms_2_steps": over_ms, "plain_ms_2_steps": plain_ms,
                              "head_groups": over_groups,
                              "note": "overlapped: the second head group's scatter runs beside the first "
                                      "group's attention; plain: scatter, barrier, attention, barrier; "
                                      "both timed after warm-up, the faster one (max over ranks) is timed"}
                             if world > 1 else None),
            "roofline_sustained": {"peak": peaks["bf16_sustained"], "frac": achieved / peaks["bf16_sustained"],
                                   "note": "measured cuBLAS bf16 GEMM held for seconds under the 1 kW cap"},
            "clocks": clk,
            "device_error": dev_err,
            "check": check,
        }
        if world > 1:
            line["all_to_all"] = {"kernel": "ulysses_scatter_kernel", "ms": a2a_ms,
                                  "nvlink_bytes_per_rank": a2a["nvlink_bytes_per_rank"],
                                  "gbs_per_direction": a2a_gbs, "peak_gbs": 770.0,
                                  "frac": a2a_gbs / 770.0,
                                  "peak_note": "measured peer copy per direction on this pool"}
            rflops = attn_flops(1, RING["heads"], RING["seq"], DIM)
            line["ring"] = {"workload": RING_WORKLOAD, "layout": ring_res["layout"], "ms_per_layer": ring_ms,
                            "tflops": rflops / (ring_ms * 1e-3) / 1e12,
                            "tokens_per_s": RING["seq"] / (ring_ms * 1e-3)}
            line["wan_ring2_full_context"] = {
                "workload": WORKLOAD + "; pure ring-2 full context: K/V gathered over NVLink, "
                            "local Q x full K/V in one call",
                "layout": f"{fc_res['pairs']} independent ring2 pairs", "ms_per_layer": fc_ms,
                "tflops_per_pair": flops / (fc_ms * 1e-3) / 1e12,
                "tflops_total": fc_res["pairs"] * flops / (fc_ms * 1e-3) / 1e12}
        cflops = attn_flops(CFG["batch"], CFG["heads"], CFG["img"] + CFG["txt"], DIM)
        line["cfg_fp8"] = {"workload": CFG_WORKLOAD, "layout": cfg_res["layout"], "ms_per_step": cfg_ms,
                           "ms_per_step_eager": cfg_ms_eager,
                           "launch": ("one CUDA graph per step (ms_per_step_eager: the same calls from Python)"
                                      if world > 1 else "the drop-in called from Python"),
                           "tflops": cflops / (cfg_ms * 1e-3) / 1e12, "accuracy": cfg_res["accuracy"]}
        if world == 1 and not args.no_cpu_baseline:
            from oracle.cpu_baseline import time_ulysses_sample

            cpu = time_ulysses_sample(SEQ, REF_SAMPLE_HEADS, DIM, world=2, steps=1, warmup=1)
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "sample")}
            line["cpu_baseline"]["kind"] = "port"
        print(json.dumps(line), flush=True)
    streamed.close()
    if not check["ok"]:
        raise SystemExit(f"the timed step's output failed its sampled fp32 check: {check}")
    if over is not None:
        over.close()
    uly.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
