"""The drop-in: a `usp_attention` callable backed by the B200 kernels.

`make_b200_usp_attention` returns a callable with the signature and typed
refusals of the reference's `usp_attention` (adapters/base.py:216-326), so
the reference's `_AttentionDispatch.configure` (actor/attention_dispatch.py:
148-251) can bind it under a new kernel name (B200_SP).  Inside:

- pure Ulysses (ring degree 1): fused scatter -> barrier -> attention with
  the inverse all-to-all in its epilogue -> barrier; a joint-order
  descriptor (adapters/usp_sequence_order.py) is applied by the scatter and
  the epilogue row maps, never by index copies;
- pad rows (adapters/usp_pad_exclusion.py:112-137): the same fused path,
  with keep bits over keys and query rows applied inside the attention
  kernel (excluded keys never enter a softmax, dropped rows are written as
  zeros) instead of index_select / zero-restore copies;
- query-group biases (adapters/usp_query_bias.py:109-130), key rows or
  per-query rectangles, added to the scaled logits inside the kernel;
- Ulysses x ring: Ulysses scatter inside the Ulysses group, ring attention
  over the ring group, inverse all-to-all kernel;
- pure ring with full_context_ring=True: the Wan Ring2 full-context strategy
  (adapters/wan_ring_full_context.py:298-449), K/V gathered into rank-major
  slots over NVLink and one local-Q x full-KV attention call, no merge.

Per-shape plans (peer windows, workspaces) are built on first use.  Every
rank issues the same calls in the same order, as the reference's
collectives require, so the window exchange on first use stays collective.
"""
from __future__ import annotations

import math

import torch

from ._lib import MAX_BIAS_GROUPS
from .comm import PeerWindows
from .ops import attention_fwd, attention_fwd_ext, keep_bits, kernel_head_dim
from .ring import FullContextRingAttention, RingAttention
from .ulysses import attention_routed, ulysses_gather, ulysses_scatter


# The head dimension the kernels run; smaller heads (multiples of 8) are
# zero-padded to it, as the capability table's limit of 128 promises.
KERNEL_HEAD_DIM = 128


class UnsupportedModelError(RuntimeError):
    """Typed refusal, the reference's adapters/base.py:37 class."""


def _mask_is_noop(mask) -> bool:
    """adapters/base.py:41-45."""
    if mask.dtype == torch.bool:
        return bool(mask.all())
    return not bool(mask.any())


def _check_pad_rows(rows: int, drop_rows) -> None:
    """Refuse pad rows outside the gathered axis before any device work
    (adapters/usp_pad_exclusion.py:93-108)."""
    if not drop_rows:
        return
    highest = max(drop_rows)
    if highest >= rows or min(drop_rows) < 0:
        raise UnsupportedModelError(
            f"a divisibility pad row at index {highest} was handed to an attention whose axis "
            f"carries {rows} rows. This is a dgx-monarch fault, not a workflow setting.")


class _Groups:
    """Ulysses and ring process groups plus each group's rank/world."""

    def __init__(self, ulysses_group, ring_group):
        import torch.distributed as dist

        self.uly_group, self.ring_group = ulysses_group, ring_group
        inited = dist.is_available() and dist.is_initialized()
        self.uly_world = dist.get_world_size(ulysses_group) if (inited and ulysses_group is not None) else 1
        self.uly_rank = dist.get_rank(ulysses_group) if (inited and ulysses_group is not None) else 0
        self.ring_world = dist.get_world_size(ring_group) if (inited and ring_group is not None) else 1
        self.ring_rank = dist.get_rank(ring_group) if (inited and ring_group is not None) else 0


class B200SequenceParallelAttention:
    """Setup-generation-bound implementation behind the callable."""

    def __init__(self, *, ulysses_group=None, ring_group=None, generation: int = 1,
                 device: torch.device | None = None, fp8: bool = False,
                 full_context_ring: bool = False) -> None:
        self.groups = _Groups(ulysses_group, ring_group)
        self.fp8 = fp8
        self.full_context_ring = full_context_ring
        self.generation = generation
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self._plans: dict = {}
        self.closed = False

    # ---------------------------------------------------------------- plans
    def _ulysses_plan(self, b, ls, h, hkv, d, dtype):
        key = ("uly", b, ls, h, hkv, d, dtype)
        plan = self._plans.get(key)
        if plan is not None:
            return plan
        g = self.groups
        p = g.uly_world
        elt = torch.empty((), dtype=dtype).element_size()
        s = ls * p
        q_bytes = b * s * (h // p) * d * elt
        kv_bytes = b * s * (hkv // p) * d * elt
        out_bytes = b * ls * h * d * elt
        win = PeerWindows(q_bytes + 2 * kv_bytes + out_bytes + 4 * 256, device=self.device,
                          group=g.uly_group, rank=g.uly_rank, world=p, generation=self.generation)
        offs = [win.carve(q_bytes), win.carve(kv_bytes), win.carve(kv_bytes), win.carve(out_bytes)]
        plan = {
            "win": win, "offs": offs,
            "recv": [win.local_tensor(offs[0], (b, s, h // p, d), dtype),
                     win.local_tensor(offs[1], (b, s, hkv // p, d), dtype),
                     win.local_tensor(offs[2], (b, s, hkv // p, d), dtype)],
            "out": win.local_tensor(offs[3], (b, ls, h, d), dtype),
        }
        if self.fp8:
            # e4m3 copies of the gathered heads and their per-head descales;
            # after the scatter each head is whole on this rank, so the absmax
            # needs no cross-rank reduction.
            plan["q8"] = torch.empty(b, s, h // p, d, device=self.device, dtype=torch.float8_e4m3fn)
            plan["k8"] = torch.empty(b, s, hkv // p, d, device=self.device, dtype=torch.float8_e4m3fn)
            plan["v8"] = torch.empty(b, s, hkv // p, d, device=self.device, dtype=torch.float8_e4m3fn)
            plan["ds"] = [torch.empty(h // p, device=self.device, dtype=torch.float32),
                          torch.empty(hkv // p, device=self.device, dtype=torch.float32),
                          torch.empty(hkv // p, device=self.device, dtype=torch.float32)]
        self._plans[key] = plan
        return plan

    def _ring_plan(self, b, lq, lk, h, hkv, d, dtype):
        key = ("ring", b, lq, lk, h, hkv, d, dtype)
        plan = self._plans.get(key)
        if plan is None:
            g = self.groups
            if self.full_context_ring and g.uly_world == 1:
                plan = FullContextRingAttention(world=g.ring_world, rank=g.ring_rank, batch=b, q_len=lq,
                                                kv_len=lk, heads=h, kv_heads=hkv, head_dim=d,
                                                device=self.device, group=g.ring_group,
                                                generation=self.generation, dtype=dtype)
            else:
                plan = RingAttention(world=g.ring_world, rank=g.ring_rank, batch=b, q_len=lq, kv_len=lk,
                                     heads=h, kv_heads=hkv, head_dim=d, device=self.device,
                                     group=g.ring_group, generation=self.generation, dtype=dtype)
            self._plans[key] = plan
        return plan

    # ---------------------------------------------------------------- forward
    def attend(self, q_l, k_l, v_l, drop_rows, kv_drop_rows, sequence_order, bias_groups=None,
               softmax_scale=None):
        """(B, Ls, H, D) local rows in, (B, Ls, H, D) local rows out.  softmax_scale
        None is 1/sqrt(D)."""
        if self.closed:
            raise UnsupportedModelError("this attention implementation belongs to a retired setup "
                                        "generation and cannot run")
        g = self.groups
        b, ls, h, d = q_l.shape
        hkv = k_l.shape[2]
        p = g.uly_world
        if h % p or hkv % p:
            raise UnsupportedModelError(
                f"{h} query / {hkv} key-value heads do not divide the Ulysses degree {p}")
        seg0 = 0
        if sequence_order is not None:
            text, image = sequence_order.text_rows, sequence_order.image_rows
            if text + image != ls or q_l.shape != k_l.shape:
                raise UnsupportedModelError(
                    "joint Ulysses order cannot preserve this attention contract: the local rows "
                    "do not tile the declared text/image pair")
            seg0 = text
            # The descriptor names stock order on the gathered axis; pad rows
            # arrive in rank-major coordinates and are remapped here.
            if drop_rows or kv_drop_rows:
                inv = _joint_inverse(text, image, p)
                drop_rows = sorted(inv[r] for r in drop_rows) if drop_rows else drop_rows
                kv_drop_rows = sorted(inv[r] for r in kv_drop_rows) if kv_drop_rows else kv_drop_rows
        _check_pad_rows(ls * p, drop_rows)
        _check_pad_rows(k_l.shape[1] * p, kv_drop_rows)
        if p == 1 and g.ring_world == 1 and not self.fp8:
            return self._local(q_l, k_l, v_l, drop_rows, kv_drop_rows, bias_groups, softmax_scale)
        if p == 1 and g.ring_world == 1:
            return self._local_fp8(q_l, k_l, v_l, drop_rows, kv_drop_rows, bias_groups, softmax_scale)
        if g.ring_world > 1:
            if self.fp8 and self.full_context_ring and p == 1:
                # adapters/wan_ring_full_context.py:10 admits fp16 and bf16 blocks only.
                raise UnsupportedModelError(
                    "the Wan Ring2 full-context path attends fp16 or bf16 blocks; run the FP8 "
                    "kernel on the rotating ring or a Ulysses topology")
            return self._hybrid(q_l, k_l, v_l, softmax_scale)
        plan = self._ulysses_plan(b, ls, h, hkv, d, q_l.dtype)
        win, offs = plan["win"], plan["offs"]
        if hkv == h:
            ulysses_scatter([q_l, k_l, v_l], [[win.peer_ptr(r, o) for r in range(p)] for o in offs[:3]],
                            world=p, rank=g.uly_rank, seg0=seg0)
        else:
            ulysses_scatter([q_l], [[win.peer_ptr(r, offs[0]) for r in range(p)]], world=p,
                            rank=g.uly_rank, seg0=seg0)
            ulysses_scatter([k_l, v_l], [[win.peer_ptr(r, o) for r in range(p)] for o in offs[1:3]],
                            world=p, rank=g.uly_rank, seg0=seg0)
        win.barrier()
        qg, kg, vg = plan["recv"]
        out_ptrs = [win.peer_ptr(r, offs[3]) for r in range(p)]
        if self.fp8:
            from .prologue import quantize_e4m3_per_head_many

            # Pad rows neither attend nor set a head's scale, as when the
            # reference hands its inner FP8 kernel the real rows only.
            q_keep = keep_bits(qg.shape[1], drop_rows, qg.device)
            k_keep = keep_bits(kg.shape[1], kv_drop_rows, qg.device)
            quantize_e4m3_per_head_many(zip((qg, kg, vg), (plan["q8"], plan["k8"], plan["v8"]), plan["ds"],
                                            (q_keep, k_keep, k_keep)))
            descales = {"q_descale": plan["ds"][0], "k_descale": plan["ds"][1], "v_descale": plan["ds"][2]}
            if not drop_rows and not kv_drop_rows and not bias_groups:
                attention_routed(plan["q8"], plan["k8"], plan["v8"], out_ptrs, (ls * h * d, h * d, d),
                                 world=p, rank=g.uly_rank, seq_local=ls, seg0=seg0,
                                 softmax_scale=softmax_scale, **descales)
            else:
                attention_fwd_ext(plan["q8"], plan["k8"], plan["v8"], key_keep=k_keep, query_keep=q_keep,
                                  bias_groups=_rank_bias(bias_groups, g.uly_rank, h // p,
                                                         kg.shape[1], kv_drop_rows),
                                  route={"o_peers": out_ptrs, "world": p, "rank": g.uly_rank,
                                         "seq_local": ls, "seg0": seg0},
                                  out_strides=(ls * h * d, h * d, d), softmax_scale=softmax_scale,
                                  **descales)
        elif not drop_rows and not kv_drop_rows and not bias_groups:
            attention_routed(qg, kg, vg, out_ptrs, (ls * h * d, h * d, d), world=p, rank=g.uly_rank,
                             seq_local=ls, seg0=seg0, softmax_scale=softmax_scale)
        else:
            # Pads and biases live on the full axis, which this rank holds for
            # its heads; the kernel applies both and still routes the output.
            attention_fwd_ext(qg, kg, vg, key_keep=keep_bits(kg.shape[1], kv_drop_rows, qg.device),
                              query_keep=keep_bits(qg.shape[1], drop_rows, qg.device),
                              bias_groups=_rank_bias(bias_groups, g.uly_rank, h // p,
                                                     kg.shape[1], kv_drop_rows),
                              route={"o_peers": out_ptrs, "world": p, "rank": g.uly_rank,
                                     "seq_local": ls, "seg0": seg0},
                              out_strides=(ls * h * d, h * d, d), softmax_scale=softmax_scale)
        win.barrier()
        return plan["out"].clone()

    def _local(self, q, k, v, drop_rows, kv_drop_rows, bias_groups=None, softmax_scale=None):
        if drop_rows or kv_drop_rows or bias_groups:
            out, _ = attention_fwd_ext(q, k, v, key_keep=keep_bits(k.shape[1], kv_drop_rows, q.device),
                                       query_keep=keep_bits(q.shape[1], drop_rows, q.device),
                                       bias_groups=_rank_bias(bias_groups, 0, q.shape[2],
                                                              k.shape[1], kv_drop_rows),
                                       softmax_scale=softmax_scale)
            return out
        out, _ = attention_fwd(q, k, v, return_lse=False, softmax_scale=softmax_scale)
        return out

    def _local_fp8(self, q, k, v, drop_rows=None, kv_drop_rows=None, bias_groups=None,
                   softmax_scale=None):
        """One rank, e4m3: quantise the caller's heads in place of a scatter
        and attend into a fresh output (no window copy, no barrier).  Pad rows
        neither attend nor set a head's scale."""
        from .prologue import quantize_e4m3_per_head_many

        b, ls, h, d = q.shape
        key = ("fp8_local", b, ls, k.shape[1], h, k.shape[2], d)
        bufs = self._plans.get(key)
        if bufs is None:
            bufs = {"q8": torch.empty(q.shape, device=self.device, dtype=torch.float8_e4m3fn),
                    "k8": torch.empty(k.shape, device=self.device, dtype=torch.float8_e4m3fn),
                    "v8": torch.empty(v.shape, device=self.device, dtype=torch.float8_e4m3fn),
                    "ds": [torch.empty(x.shape[2], device=self.device, dtype=torch.float32) for x in (q, k, v)]}
            self._plans[key] = bufs
        q_keep = keep_bits(q.shape[1], drop_rows, q.device)
        k_keep = keep_bits(k.shape[1], kv_drop_rows, q.device)
        quantize_e4m3_per_head_many(zip((q, k, v), (bufs["q8"], bufs["k8"], bufs["v8"]), bufs["ds"],
                                        (q_keep, k_keep, k_keep)))
        descales = {"q_descale": bufs["ds"][0], "k_descale": bufs["ds"][1], "v_descale": bufs["ds"][2]}
        if drop_rows or kv_drop_rows or bias_groups:
            out, _ = attention_fwd_ext(bufs["q8"], bufs["k8"], bufs["v8"], key_keep=k_keep, query_keep=q_keep,
                                       bias_groups=_rank_bias(bias_groups, 0, q.shape[2], k.shape[1],
                                                              kv_drop_rows),
                                       softmax_scale=softmax_scale, **descales)
            return out
        out, _ = attention_fwd(bufs["q8"], bufs["k8"], bufs["v8"], return_lse=False,
                               softmax_scale=softmax_scale, **descales)
        return out

    def _hybrid(self, q_l, k_l, v_l, softmax_scale=None):
        """Ulysses inside the Ulysses group, ring across the ring group."""
        g = self.groups
        b, ls, h, d = q_l.shape
        hkv = k_l.shape[2]
        p = g.uly_world
        if p > 1:
            plan = self._ulysses_plan(b, ls, h, hkv, d, q_l.dtype)
            win, offs = plan["win"], plan["offs"]
            ulysses_scatter([q_l], [[win.peer_ptr(r, offs[0]) for r in range(p)]], world=p, rank=g.uly_rank)
            ulysses_scatter([k_l, v_l], [[win.peer_ptr(r, o) for r in range(p)] for o in offs[1:3]],
                            world=p, rank=g.uly_rank)
            win.barrier()
            qg, kg, vg = plan["recv"]
        else:
            qg, kg, vg = q_l, k_l, v_l
        if self.fp8:
            # Each rank quantises its query rows and its own K/V block with
            # per-head scales over exactly those rows; a block rotates with its
            # scales, so every ring step attends under the scales an inner FP8
            # kernel called on that block would take.
            from .prologue import quantize_e4m3_per_head_many

            ring = self._ring_plan(b, qg.shape[1], kg.shape[1], qg.shape[2], kg.shape[2], d,
                                   torch.float8_e4m3fn)
            (q8, qs), (k8, ks), (v8, vs) = quantize_e4m3_per_head_many((t, None, None, None) for t in (qg, kg, vg))
            out_g, _ = ring.forward(q8, k8, v8, softmax_scale=softmax_scale, q_descale=qs, k_descale=ks,
                                    v_descale=vs)
        else:
            ring = self._ring_plan(b, qg.shape[1], kg.shape[1], qg.shape[2], kg.shape[2], d, q_l.dtype)
            out_g, _ = ring.forward(qg, kg, vg, softmax_scale=softmax_scale)
        if p == 1:
            return out_g
        ulysses_gather(out_g, [win.peer_ptr(r, offs[3]) for r in range(p)], world=p, rank=g.uly_rank,
                       seq_local=ls, heads=h)
        win.barrier()
        return plan["out"].clone()

    def invalidate(self) -> None:
        """Release every window bound to this generation
        (actor/attention_dispatch.py:383-401)."""
        for plan in self._plans.values():
            if isinstance(plan, dict):
                if "win" in plan:
                    plan["win"].close()
            else:
                plan.close()
        self._plans.clear()
        self.closed = True


def _rank_bias(groups, rank: int, heads_local: int, keys: int, kv_drop_rows):
    """This rank's slice of the group biases: (B|1, H|1, Q|1, K') -> fp32
    (B|1, H_local|1, Q|1, K'') for the heads the rank attends after the scatter.

    A bias names keys by their position among the kept keys
    (adapters/usp_query_bias.py:95-106 runs after the pads are dropped).  The
    kernel reads the padded axis, so where a pad key precedes a declared key
    the bias is spread onto the kept positions; pads at the tail need no
    change, and a zero column adds nothing where the bias declared no key."""
    if not groups:
        return None
    kept = None
    if kv_drop_rows:
        drop = sorted(set(kv_drop_rows))
        if drop != list(range(keys - len(drop), keys)):
            dropped = set(drop)
            kept = [r for r in range(keys) if r not in dropped]
    out = []
    for start, end, bias in groups:
        if bias is None:
            out.append((start, end, None))
            continue
        bb = bias
        if bb.shape[1] > 1:
            bb = bb[:, rank * heads_local:(rank + 1) * heads_local]
        bb = bb.float()
        if kept is not None:
            n = bb.shape[3]
            index = torch.tensor(kept[:n], device=bb.device)
            spread = bb.new_zeros((*bb.shape[:3], kept[n - 1] + 1 if n else 0))
            spread.index_copy_(3, index, bb)
            bb = spread
        out.append((start, end, bb.contiguous()))
    return out


def validate_bias_groups(groups, queries: int, keys: int, batch: int, heads: int) -> None:
    """The partition contract of adapters/usp_query_bias.py:64-97, plus the
    broadcast and group-count limits of the kernel."""
    cursor = 0
    for start, end, bias in groups:
        if start != cursor or end < start or end > queries:
            raise UnsupportedModelError(
                f"query bias groups are malformed: group [{start}, {end}) does not continue the "
                f"partition of [0, {queries}) at row {cursor}")
        cursor = end
        if bias is None:
            continue
        if bias.ndim != 4 or bias.shape[2] not in (1, end - start):
            raise UnsupportedModelError(
                f"query bias groups are malformed: a bias shaped {tuple(bias.shape)} does not "
                f"broadcast over the {end - start} query rows of its group as (B, H, Q, K)")
        if bias.shape[3] > keys:
            raise UnsupportedModelError(
                f"query bias groups are malformed: a bias declares {bias.shape[3]} keys over a "
                f"sequence of {keys}")
        if bias.shape[0] not in (1, batch) or bias.shape[1] not in (1, heads):
            raise UnsupportedModelError(
                f"query bias groups are malformed: a bias shaped {tuple(bias.shape)} does not "
                f"broadcast over batch {batch} and {heads} heads")
    if cursor != queries:
        raise UnsupportedModelError(
            f"query bias groups are malformed: the groups cover {cursor} of {queries} query rows")
    biased = sum(1 for group in groups if group[2] is not None)
    if biased > MAX_BIAS_GROUPS:
        raise UnsupportedModelError(
            f"the B200 kernel applies at most {MAX_BIAS_GROUPS} biased query groups in one call; "
            f"this one carries {biased}. Select TORCH_FLASH for it.")


def _joint_inverse(text: int, image: int, world: int) -> list[int]:
    """rank-major row -> canonical row (adapters/usp_sequence_order.py:69-78)."""
    local = text + image
    inv = [0] * (local * world)
    canon = 0
    for r in range(world):
        for t in range(text):
            inv[r * local + t] = canon
            canon += 1
    for r in range(world):
        for i in range(image):
            inv[r * local + text + i] = canon
            canon += 1
    return inv


def make_b200_usp_attention(*, ulysses_group=None, ring_group=None, generation: int = 1,
                            device: torch.device | None = None, fp8: bool = False,
                            full_context_ring: bool = False):
    """A callable with the reference's usp_attention contract
    (adapters/base.py:216-326) on the B200 kernels.  fp8=True quantises the
    gathered heads to e4m3 with per-head absmax scales and runs the FP8
    tensor-core path (output bf16).  full_context_ring=True runs pure ring
    topologies as the Wan Ring2 full-context path (one attention call over
    the gathered K/V) instead of the rotating ring with an LSE merge."""
    impl = B200SequenceParallelAttention(ulysses_group=ulysses_group, ring_group=ring_group,
                                         generation=generation, device=device, fp8=fp8,
                                         full_context_ring=full_context_ring)

    def usp_attention(q, k, v, heads, mask=None, attn_precision=None,
                      skip_reshape=False, skip_output_reshape=False,
                      enable_gqa=False, drop_rows=None, kv_drop_rows=None,
                      query_bias_groups=None, sequence_order=None, **kwargs):
        if mask is not None and not _mask_is_noop(mask):
            raise UnsupportedModelError(
                "this render carries a non-trivial attention mask, which the sharded attention "
                "kernel cannot apply. Run it on a cfg or single topology; a USP render that "
                "dropped it would be silently wrong (docs/MODELS.md).")
        if skip_reshape:
            if any(t.ndim != 4 for t in (q, k, v)):
                raise UnsupportedModelError("skip_reshape attention requires q/k/v shaped (B, H, L, D)")
            b, h, _, d = q.shape
            if h != heads:
                raise UnsupportedModelError(f"attention declared {heads} query heads but q carries {h}")
            if k.shape[0] != b or v.shape[0] != b or k.shape[-1] != d or v.shape[-1] != d:
                raise UnsupportedModelError("q/k/v batch and head dimensions must agree before USP attention")
            q_l, k_l, v_l = (t.transpose(1, 2) for t in (q, k, v))
        else:
            if any(t.ndim != 3 for t in (q, k, v)):
                raise UnsupportedModelError("attention requires q/k/v shaped (B, L, H*D)")
            b, _, inner = q.shape
            h = heads
            if inner % h:
                raise UnsupportedModelError(f"query inner dimension {inner} is not divisible by {h} heads")
            d = inner // h
            if k.shape[0] != b or v.shape[0] != b:
                raise UnsupportedModelError("q/k/v batch dimensions must agree")

            def _reshape(t, name):
                if t.shape[-1] % d:
                    raise UnsupportedModelError(
                        f"{name} inner dimension {t.shape[-1]} is not divisible by head dimension {d}")
                return t.reshape(b, -1, t.shape[-1] // d, d)

            q_l = q.reshape(b, -1, h, d)
            k_l = _reshape(k, "key")
            v_l = _reshape(v, "value")
        head_dim = q_l.shape[-1]
        if head_dim > KERNEL_HEAD_DIM or head_dim % 8:
            raise UnsupportedModelError(
                f"head_dim {head_dim}: the B200 sequence-parallel kernels carry head dimensions up "
                f"to {KERNEL_HEAD_DIM} in multiples of 8")
        kv_heads = k_l.shape[2]
        if v_l.shape[2] != kv_heads:
            raise UnsupportedModelError(f"key/value head counts differ ({kv_heads} vs {v_l.shape[2]})")
        if kv_heads != h:
            if not enable_gqa:
                raise UnsupportedModelError(
                    f"attention has {h} query heads and {kv_heads} K/V heads but did not set enable_gqa=True")
            if h % kv_heads:
                raise UnsupportedModelError(
                    f"GQA query heads ({h}) must be divisible by K/V heads ({kv_heads})")
            if kv_heads % impl.groups.uly_world:
                # The kernel maps query heads to shared K/V heads natively, and
                # the ring rotates the shared K/V heads alone; only a K/V head
                # count the Ulysses degree cannot split is expanded.
                rep = h // kv_heads
                k_l = k_l.repeat_interleave(rep, dim=2)
                v_l = v_l.repeat_interleave(rep, dim=2)
        if kwargs:
            raise UnsupportedModelError(
                f"the B200 sequence-parallel kernel cannot apply extra attention arguments {sorted(kwargs)}")
        padded = bool(drop_rows) or bool(kv_drop_rows)
        ring_world = impl.groups.ring_world
        if padded and ring_world > 1:
            raise UnsupportedModelError(
                "this sequence length needs divisibility padding, and the exact pad exclusion is "
                "ulysses-only; ring/hybrid attention would attend the synthetic pad rows. Use a "
                "uly* or single topology (docs/ADAPTERS.md).")
        if query_bias_groups:
            if ring_world != 1:
                raise UnsupportedModelError(
                    "this render biases attention between token groups, and ring or hybrid "
                    "attention shards the key axis, so the weights cannot be applied where the "
                    "kernel reads them. Use a pure-ulysses topology.")
            if sequence_order is not None:
                raise UnsupportedModelError(
                    "joint Ulysses order cannot preserve this attention contract: query-bias group "
                    "coordinates are present")
            full_q = q_l.shape[1] * impl.groups.uly_world
            full_k = k_l.shape[1] * impl.groups.uly_world
            if drop_rows:
                tail = list(range(full_q - len(drop_rows), full_q))
                if list(drop_rows) != tail:
                    raise UnsupportedModelError(
                        f"a query-group bias met {len(drop_rows)} divisibility pad row(s) away from "
                        f"the tail of its {full_q}-row sequence, where the group boundaries stop "
                        "being exact.")
            validate_bias_groups(query_bias_groups, full_q - len(drop_rows or ()),
                                 full_k - len(kv_drop_rows if kv_drop_rows is not None else drop_rows or ()),
                                 b, h)
        if sequence_order is not None and ring_world != 1:
            sequence_order = None
        # The kernels compute in the caller's 16-bit format: fp16 models stay in
        # fp16 (the reference's flash path takes fp16 and bf16 alike), bf16 in
        # bf16.  fp32 callers -- and every caller of the e4m3 path, whose
        # quantiser reads bf16 -- are rounded to bf16; the output returns in
        # the caller's dtype.
        compute = q_l.dtype if q_l.dtype in (torch.float16, torch.bfloat16) else torch.bfloat16
        if impl.fp8:
            compute = torch.bfloat16
        if q_l.dtype != compute or k_l.dtype != compute or v_l.dtype != compute:
            q_l, k_l, v_l = (t.to(compute) for t in (q_l, k_l, v_l))
        dk = kernel_head_dim(head_dim, fp8=impl.fp8, ring=impl.groups.ring_world > 1)
        if head_dim < dk:
            # Zero columns add exact zeros to every logit and give zero output
            # columns; the scale stays that of the real head dimension.
            q_l, k_l, v_l = (torch.nn.functional.pad(t, (0, dk - head_dim)) for t in (q_l, k_l, v_l))
        q_l, k_l, v_l = (t if t.stride(-1) == 1 else t.contiguous() for t in (q_l, k_l, v_l))
        kv_rows = drop_rows if kv_drop_rows is None else kv_drop_rows
        out = impl.attend(q_l, k_l, v_l, drop_rows, kv_rows, sequence_order, query_bias_groups,
                          softmax_scale=1.0 / math.sqrt(head_dim))
        if head_dim < dk:
            out = out[..., :head_dim]
        out = out.to(q.dtype)
        if skip_output_reshape:
            return out.transpose(1, 2)
        return out.reshape(b, -1, h * d)

    usp_attention.impl = impl
    return usp_attention
