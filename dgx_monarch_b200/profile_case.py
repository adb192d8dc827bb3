"""Representative launches of the library's kernels, for profiler captures.

    python -m dgx_monarch_b200.profile_case SEQ HEADS [CHUNKS]  # bf16 attention, three launches
    python -m dgx_monarch_b200.profile_case fp8 SEQ HEADS       # e4m3 attention, three launches
    python -m dgx_monarch_b200.profile_case kernels             # every other kernel, one GPU

CHUNKS selects the release of P in 1, 2 or 4 chunks per block (ops.set_p_chunks).

The `kernels` cases use the C2 (Flux/Krea2 block) and C4 shapes on one rank,
each input larger than the 126 MB L2 where the kernel is HBM-bound, and a few
GB of device memory in all.
"""
import sys

import torch


def attention(seq: int, heads: int, chunks: int = 0) -> None:
    from dgx_monarch_b200.ops import attention_fwd, set_p_chunks

    set_p_chunks(chunks)
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(1, seq, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    out = torch.empty_like(q)
    for _ in range(3):
        attention_fwd(q, k, v, out=out, return_lse=False)
    torch.cuda.synchronize()


def attention_fp8(seq: int, heads: int) -> None:
    """e4m3 inputs with per-head descales (the C3 path), bf16 output."""
    from dgx_monarch_b200.ops import attention_fwd
    from dgx_monarch_b200.prologue import quantize_e4m3_per_head

    g = torch.Generator(device="cuda").manual_seed(0)
    q8, k8, v8 = (quantize_e4m3_per_head(torch.randn(1, seq, heads, 128, device="cuda", generator=g).bfloat16())
                  for _ in range(3))
    out = torch.empty(1, seq, heads, 128, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        attention_fwd(q8[0], k8[0], v8[0], q_descale=q8[1], k_descale=k8[1], v_descale=v8[1], out=out,
                      return_lse=False)
    torch.cuda.synchronize()


def kernels() -> None:
    from dgx_monarch_b200 import _lib
    from dgx_monarch_b200.cfg import cfg_combine
    from dgx_monarch_b200.ops import lse_merge
    from dgx_monarch_b200.prologue import (qkv_gemm_prologue_scatter, qkv_prologue_scatter,
                                           quantize_e4m3_per_head, rope_table)
    from dgx_monarch_b200.shard import SequenceGather, SharedActivationScale

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    hid, heads, rows = 3072, 24, 9728                     # C2 on one rank
    w = lambda *s, sc=0.02: (sc * torch.randn(*s, device=dev, generator=g)).bfloat16()
    x = w(rows, hid, sc=1.0)
    wq, bq = w(3 * hid, hid), w(3 * hid)
    nq, nk = (1 + w(128)).contiguous(), (1 + w(128)).contiguous()
    pos = torch.stack((torch.zeros(rows, device=dev, dtype=torch.long),
                       torch.arange(rows, device=dev) // 96, torch.arange(rows, device=dev) % 96), dim=1)
    table = rope_table(pos, [16, 56, 56])
    recv = [torch.empty(rows, heads, 128, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    dst = [[t.data_ptr()] for t in recv]
    for _ in range(2):  # the fused QKV projection + QKNorm + RoPE + scatter
        qkv_gemm_prologue_scatter(x, wq, dst, world=1, rank=0, seq_local=rows, bias=bq,
                                  norm_mode=_lib.NORM_HEAD, norm_q_w=nq, norm_k_w=nk, rope=table)
    qkv = (x @ wq.t()).view(1, rows, 3, heads, 128)
    for _ in range(2):  # the prologue kernel on cuBLAS output
        qkv_prologue_scatter(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], dst, world=1, rank=0,
                             norm_mode=_lib.NORM_HEAD, norm_q_w=nq, norm_k_w=nk, rope=table)
    del qkv
    # The joint scatter with replicated text (512 text rows, 9216 image rows,
    # one rank): the image scatter and the text head-slice copy.
    from dgx_monarch_b200.ulysses import ulysses_scatter_joint

    txt_rows = 512
    joint = [torch.empty(1, rows, heads, 128, device=dev, dtype=torch.bfloat16)  # text + image rows
             for _ in range(3)]
    img = [w(1, rows - txt_rows, heads, 128, sc=1.0) for _ in range(3)]
    txt = [w(1, txt_rows, heads, 128, sc=1.0) for _ in range(3)]
    for _ in range(2):
        ulysses_scatter_joint(img, txt, [[t.data_ptr()] for t in joint], world=1, rank=0)
    del joint, img, txt
    # FP8 quantisation of one gathered head slab (C3: 4608 tokens x 24 heads).
    xq = torch.randn(1, 32768, 24, 128, device=dev, generator=g).bfloat16()
    for _ in range(2):
        quantize_e4m3_per_head(xq)
    # LSE merge of two ring partials (fp32, 1 x 32768 x 8 x 128).
    parts = [torch.randn(1, 32768, 8, 128, device=dev, generator=g) for _ in range(2)]
    lses = [torch.randn(1, 8, 32768, device=dev, generator=g) for _ in range(2)]
    for _ in range(2):
        lse_merge(parts, lses)
    # CFG combine of two fp32 predictions (2 x 268 MB).
    c, u = (torch.randn(64 * 1024 * 1024, device=dev, generator=g) for _ in range(2))
    for _ in range(2):
        cfg_combine(c, u, 4.0)
    del c, u
    # Shared NVFP4 activation scale over a (9728, 9216) bf16 activation, one rank.
    act = w(rows, 3 * hid, sc=1.0)
    scale = SharedActivationScale(device=dev, generation=90)
    for _ in range(2):
        scale(act)
    scale.close()
    # sp_gather of a (2, 9728, 3072) bf16 token stream, one rank.
    gather = SequenceGather(device=dev, generation=91)
    tokens = w(2, rows, hid, sc=1.0)
    for _ in range(2):
        gather(tokens, rows)
    gather.close()
    torch.cuda.synchronize()


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "kernels":
        kernels()
    elif len(sys.argv) > 1 and sys.argv[1] == "fp8":
        seq, heads = (int(sys.argv[2]), int(sys.argv[3])) if len(sys.argv) > 3 else (32768, 8)
        attention_fp8(seq, heads)
    else:
        seq, heads = (int(sys.argv[1]), int(sys.argv[2])) if len(sys.argv) > 2 else (32768, 8)
        attention(seq, heads, int(sys.argv[3]) if len(sys.argv) > 3 else 0)
