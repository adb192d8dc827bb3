"""The drop-in: a `usp_attention` callable backed by the B200 kernels.

`make_b200_usp_attention` returns a callable with the signature and typed
refusals of the reference's `usp_attention` (adapters/base.py:216-326), so
the reference's `_AttentionDispatch.configure` (actor/attention_dispatch.py:
148-251) can bind it under a new kernel name (B200_SP).  Inside:

- pure Ulysses (ring degree 1): fused scatter -> barrier -> attention with
  the inverse all-to-all in its epilogue -> barrier; a joint-order
  descriptor (adapters/usp_sequence_order.py) is applied by the scatter and
  the epilogue row maps, never by index copies;
- pad rows (adapters/usp_pad_exclusion.py:152-177): scatter, keep-index
  compaction at the full-axis point, attention, zero-restore, inverse
  all-to-all kernel;
- Ulysses x ring: Ulysses scatter inside the Ulysses group, ring attention
  over the ring group, inverse all-to-all kernel.

Per-shape plans (peer windows, workspaces) are built on first use.  Every
rank issues the same calls in the same order, as the reference's
collectives require, so the window exchange on first use stays collective.
"""
from __future__ import annotations

import math

import torch

from .comm import PeerWindows
from .ops import attention_fwd
from .ring import RingAttention
from .ulysses import attention_routed, ulysses_gather, ulysses_scatter


class UnsupportedModelError(RuntimeError):
    """Typed refusal, the reference's adapters/base.py:37 class."""


def _mask_is_noop(mask) -> bool:
    """adapters/base.py:41-45."""
    if mask.dtype == torch.bool:
        return bool(mask.all())
    return not bool(mask.any())


def _kept_rows(rows: int, drop_rows, device) -> torch.Tensor | None:
    """Ascending kept indices, built on the device; refuses out-of-range rows
    before any device scatter (adapters/usp_pad_exclusion.py:79-126)."""
    if not drop_rows:
        return None
    highest = max(drop_rows)
    if highest >= rows or min(drop_rows) < 0:
        raise UnsupportedModelError(
            f"a divisibility pad row at index {highest} was handed to an attention whose axis "
            f"carries {rows} rows. This is a dgx-monarch fault, not a workflow setting.")
    mask = torch.ones(rows, dtype=torch.bool)
    mask[sorted(set(drop_rows))] = False
    return torch.nonzero(mask).flatten().to(device)


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
                 device: torch.device | None = None, fp8: bool = False) -> None:
        self.groups = _Groups(ulysses_group, ring_group)
        self.fp8 = fp8
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
            plan = RingAttention(world=g.ring_world, rank=g.ring_rank, batch=b, q_len=lq, kv_len=lk,
                                 heads=h, kv_heads=hkv, head_dim=d, device=self.device,
                                 group=g.ring_group, generation=self.generation, dtype=dtype)
            self._plans[key] = plan
        return plan

    # ---------------------------------------------------------------- forward
    def attend(self, q_l, k_l, v_l, drop_rows, kv_drop_rows, sequence_order):
        """(B, Ls, H, D) local rows in, (B, Ls, H, D) local rows out."""
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
        if p == 1 and g.ring_world == 1 and not self.fp8:
            return self._local(q_l, k_l, v_l, drop_rows, kv_drop_rows)
        if self.fp8 and (g.ring_world > 1 or drop_rows or kv_drop_rows):
            raise UnsupportedModelError(
                "the B200 FP8 attention path runs pure Ulysses without pad rows; use the bf16 "
                "kernel for ring topologies or padded sequences")
        if g.ring_world > 1:
            return self._hybrid(q_l, k_l, v_l)
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
            from .prologue import quantize_e4m3_per_head

            for src, dst, ds in zip((qg, kg, vg), (plan["q8"], plan["k8"], plan["v8"]), plan["ds"]):
                quantize_e4m3_per_head(src, out=dst, descale=ds)
            attention_routed(plan["q8"], plan["k8"], plan["v8"], out_ptrs, (ls * h * d, h * d, d),
                             world=p, rank=g.uly_rank, seq_local=ls, seg0=seg0,
                             q_descale=plan["ds"][0], k_descale=plan["ds"][1], v_descale=plan["ds"][2])
        elif not drop_rows and not kv_drop_rows:
            attention_routed(qg, kg, vg, out_ptrs, (ls * h * d, h * d, d), world=p, rank=g.uly_rank,
                             seq_local=ls, seg0=seg0)
        else:
            full = self._exact_without_pads(qg, kg, vg, drop_rows, kv_drop_rows)
            ulysses_gather(full, out_ptrs, world=p, rank=g.uly_rank, seq_local=ls, heads=h, seg0=seg0)
        win.barrier()
        return plan["out"].clone()

    def _local(self, q, k, v, drop_rows, kv_drop_rows):
        if drop_rows or kv_drop_rows:
            return self._exact_without_pads(q, k, v, drop_rows, kv_drop_rows)
        out, _ = attention_fwd(q, k, v, return_lse=False)
        return out

    def _exact_without_pads(self, q, k, v, drop_rows, kv_drop_rows):
        """Attend the real rows only and write zeros where pads sat
        (adapters/usp_pad_exclusion.py:152-177)."""
        qi = _kept_rows(q.shape[1], drop_rows, q.device)
        if kv_drop_rows is drop_rows and k.shape[1] == q.shape[1]:
            ki = qi
        else:
            ki = _kept_rows(k.shape[1], kv_drop_rows, k.device)
        qq = q if qi is None else q.index_select(1, qi)
        kk = k if ki is None else k.index_select(1, ki)
        vv = v if ki is None else v.index_select(1, ki)
        out, _ = attention_fwd(qq, kk, vv, return_lse=False)
        if qi is None:
            return out
        full = q.new_zeros(q.shape)
        full[:, qi] = out
        return full

    def _hybrid(self, q_l, k_l, v_l):
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
        ring = self._ring_plan(b, qg.shape[1], kg.shape[1], qg.shape[2], kg.shape[2], d, q_l.dtype)
        out_g, _ = ring.forward(qg, kg, vg)
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
                plan["win"].close()
            else:
                plan.close()
        self._plans.clear()
        self.closed = True


def _joint_inverse(text: int, image: int, world: int) -> list[int]:
    """rank-major row -> canonical row (adapters/usp_sequence_order.py:246-261)."""
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
                            device: torch.device | None = None, fp8: bool = False):
    """A callable with the reference's usp_attention contract
    (adapters/base.py:216-326) on the B200 kernels.  fp8=True quantises the
    gathered heads to e4m3 with per-head absmax scales and runs the FP8
    tensor-core path (output bf16)."""
    impl = B200SequenceParallelAttention(ulysses_group=ulysses_group, ring_group=ring_group,
                                         generation=generation, device=device, fp8=fp8)

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
            if kv_heads % impl.groups.uly_world or impl.groups.ring_world > 1:
                # The kernel maps query heads to shared K/V heads natively; only a
                # K/V head count the Ulysses degree cannot split is expanded.
                rep = h // kv_heads
                k_l = k_l.repeat_interleave(rep, dim=2)
                v_l = v_l.repeat_interleave(rep, dim=2)
        if kwargs:
            raise UnsupportedModelError(
                f"the B200 sequence-parallel kernel cannot apply extra attention arguments {sorted(kwargs)}")
        if query_bias_groups:
            raise UnsupportedModelError(
                "query-group attention bias is not supported by the B200 sequence-parallel kernel; "
                "select TORCH_FLASH for this family")
        padded = bool(drop_rows) or bool(kv_drop_rows)
        ring_world = impl.groups.ring_world
        if padded and ring_world > 1:
            raise UnsupportedModelError(
                "this sequence length needs divisibility padding, and the exact pad exclusion is "
                "ulysses-only; ring/hybrid attention would attend the synthetic pad rows. Use a "
                "uly* or single topology (docs/ADAPTERS.md).")
        if sequence_order is not None and ring_world != 1:
            sequence_order = None
        if q_l.dtype != torch.bfloat16:
            q_l, k_l, v_l = (t.to(torch.bfloat16) for t in (q_l, k_l, v_l))
        q_l, k_l, v_l = (t if t.stride(-1) == 1 else t.contiguous() for t in (q_l, k_l, v_l))
        kv_rows = drop_rows if kv_drop_rows is None else kv_drop_rows
        out = impl.attend(q_l, k_l, v_l, drop_rows, kv_rows, sequence_order)
        out = out.to(q.dtype)
        if skip_output_reshape:
            return out.transpose(1, 2)
        return out.reshape(b, -1, h * d)

    usp_attention.impl = impl
    return usp_attention
