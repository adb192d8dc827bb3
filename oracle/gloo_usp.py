"""The reference's Ulysses/ring data path restated over a real process group.

TEST INFRASTRUCTURE ONLY -- the oracle (see oracle/__init__.py).  Each rank
runs the third-party leaves the reference calls as CPU code over
torch.distributed (gloo):

- SeqAllToAll4D(pg, x, 2, 1) / (pg, x, 1, 2) as all_to_all_single with the
  rank-major gathered order (adapters/usp_full_axis.py:27-29,40);
- ring attention as P2P rotation of K/V blocks plus an LSE merge
  (the path reached from adapters/base.py:320);
- joint image+text attention with the text replicated on every rank: the
  image shards go through the all-to-all, each rank head-slices its full text
  locally, and the text output is all-gathered over heads.

The inner kernel is torch SDPA math in fp32 (what the reference's ATen SDPA
computes, adapters/wan_ring_full_context.py:160-167).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def attention_lse_torch(q, k, v, scale=None):
    """fp32/fp64 torch attention, (B, L, H, D) -> out (B, L, H, D), lse (B, H, L)."""
    scale = scale or 1.0 / math.sqrt(q.shape[-1])
    qh, kh, vh = (t.transpose(1, 2) for t in (q, k, v))
    logits = torch.matmul(qh, kh.transpose(-1, -2)) * scale
    lse = torch.logsumexp(logits, dim=-1)
    out = torch.matmul(torch.softmax(logits, dim=-1), vh)
    return out.transpose(1, 2), lse


def seq_all_to_all_4d(x: torch.Tensor, scatter_dim: int, gather_dim: int, group=None) -> torch.Tensor:
    """yunchang SeqAllToAll4D semantics over `group` with all_to_all_single."""
    world = dist.get_world_size(group)
    if world == 1:
        return x
    if (scatter_dim, gather_dim) == (2, 1):
        b, ls, h, d = x.shape
        hl = h // world
        # (B, Ls, P, Hl, D) -> (P, Ls, B, Hl, D): chunk r goes to rank r.
        send = x.reshape(b, ls, world, hl, d).permute(2, 1, 0, 3, 4).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
        # recv[s] = source s's rows -> rank-major concat along the sequence.
        return recv.permute(2, 0, 1, 3, 4).reshape(b, world * ls, hl, d).contiguous()
    if (scatter_dim, gather_dim) == (1, 2):
        b, s, hl, d = x.shape
        ls = s // world
        send = x.reshape(b, world, ls, hl, d).permute(1, 0, 2, 3, 4).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
        # recv[src] = src's head slice for my rows -> heads ordered by source.
        return recv.permute(1, 2, 0, 3, 4).reshape(b, ls, world * hl, d).contiguous()
    raise ValueError((scatter_dim, gather_dim))


def ulysses_attention(q, k, v, group=None, scale=None):
    """Pure Ulysses over `group`: (B, Ls, H, D) local rows in, same out."""
    qg, kg, vg = (seq_all_to_all_4d(t, 2, 1, group) for t in (q, k, v))
    out, _ = attention_lse_torch(qg, kg, vg, scale)
    return seq_all_to_all_4d(out, 1, 2, group)


def ulysses_joint_attention(q_img, k_img, v_img, q_txt, k_txt, v_txt, group=None, scale=None,
                            text_first=True):
    """Joint attention with image rows sharded and text rows replicated.

    Returns (image output rows of this rank (B, Ls, H, D), full text output
    (B, T, H, D)).  Keys are ordered [text, image] (text_first) or
    [image, text], matching the unsharded concatenation.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    h = q_img.shape[2]
    hl = h // world
    qi, ki, vi = (seq_all_to_all_4d(t, 2, 1, group) for t in (q_img, k_img, v_img))
    qt, kt, vt = (t[:, :, rank * hl:(rank + 1) * hl] for t in (q_txt, k_txt, v_txt))
    t_rows = q_txt.shape[1]
    if text_first:
        q, k, v = (torch.cat(p, dim=1) for p in ((qt, qi), (kt, ki), (vt, vi)))
    else:
        q, k, v = (torch.cat(p, dim=1) for p in ((qi, qt), (ki, kt), (vi, vt)))
    out, _ = attention_lse_torch(q, k, v, scale)
    if text_first:
        out_t, out_i = out[:, :t_rows], out[:, t_rows:]
    else:
        out_i, out_t = out[:, :-t_rows], out[:, -t_rows:]
    img = seq_all_to_all_4d(out_i.contiguous(), 1, 2, group)
    parts = [torch.empty_like(out_t.contiguous()) for _ in range(world)]
    dist.all_gather(parts, out_t.contiguous(), group=group)
    return img, torch.cat(parts, dim=2)


def ring_attention(q, k, v, group=None, scale=None):
    """Ring over `group`: K/V blocks rotate by P2P, partial results merge by LSE."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    outs, lses = [], []
    kc, vc = k.contiguous(), v.contiguous()
    for step in range(world):
        o, l = attention_lse_torch(q, kc, vc, scale)
        outs.append(o)
        lses.append(l)
        if step == world - 1:
            break
        nk, nv = torch.empty_like(kc), torch.empty_like(vc)
        nxt = dist.get_global_rank(group, (rank + 1) % world) if group is not None else (rank + 1) % world
        prv = dist.get_global_rank(group, (rank - 1) % world) if group is not None else (rank - 1) % world
        ops = [dist.P2POp(dist.isend, kc, nxt, group), dist.P2POp(dist.isend, vc, nxt, group),
               dist.P2POp(dist.irecv, nk, prv, group), dist.P2POp(dist.irecv, nv, prv, group)]
        for req in dist.batch_isend_irecv(ops):
            req.wait()
        kc, vc = nk, nv
    lse_all = torch.stack(lses)
    lse = torch.logsumexp(lse_all, dim=0)
    out = torch.zeros_like(outs[0])
    for o, l in zip(outs, lses):
        out += torch.exp(l - lse).transpose(1, 2).unsqueeze(-1) * o
    return out, lse
