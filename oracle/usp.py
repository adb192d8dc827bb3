"""CPU restatement of the reference's USP attention algebra (numpy / float64).

TEST INFRASTRUCTURE ONLY -- the oracle.  See oracle/__init__.py for who may
import it.  Each function cites the reference file:line it restates (paths
inside the dgx-monarch source tree, src/dgx_monarch/...).

Array layout follows the reference: token tensors are (B, L, ...) with the
sequence on axis 1; attention tensors are (B, L, H, D).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


class OracleRefusal(RuntimeError):
    """Stands in for the reference's UnsupportedModelError (adapters/base.py:37)."""


# ----------------------------------------------------------------- sharding
def pad_seq_to_multiple(x: np.ndarray, multiple: int, axis: int = 1) -> tuple[np.ndarray, int]:
    """Zero-pad `axis` up to a multiple (adapters/base.py:48-56)."""
    orig = x.shape[axis]
    short = (multiple - orig % multiple) % multiple
    if short == 0:
        return x, orig
    pad = [(0, 0)] * x.ndim
    pad[axis] = (0, short)
    return np.pad(x, pad), orig


def shard_seq(x: np.ndarray, world: int, rank: int, axis: int = 1,
              allow_padding: bool = True) -> tuple[np.ndarray, int]:
    """This rank's contiguous chunk after padding to the SP degree
    (adapters/base.py:91-123; torch.chunk semantics on an evenly divisible axis)."""
    orig = x.shape[axis]
    if orig % world:
        if not allow_padding:
            raise OracleRefusal(f"length {orig} on dim {axis} is not divisible by {world}")
        x, _ = pad_seq_to_multiple(x, world, axis)
    step = x.shape[axis] // world
    index = [slice(None)] * x.ndim
    index[axis] = slice(rank * step, (rank + 1) * step)
    return x[tuple(index)], orig


def sp_gather(chunks: list[np.ndarray], orig_len: int, axis: int = 1) -> np.ndarray:
    """All-gather of sequence chunks, then trim (adapters/base.py:126-131)."""
    full = np.concatenate(chunks, axis=axis)
    index = [slice(None)] * full.ndim
    index[axis] = slice(0, orig_len)
    return full[tuple(index)]


def padded_row_indices(segments: list[tuple[int, int]], world: int) -> list[int]:
    """Gathered (rank-major) coordinates of shard_seq's pad rows
    (adapters/base.py:134-149)."""
    chunk = sum(local for _, local in segments)
    rows: list[int] = []
    offset = 0
    for orig, local in segments:
        for padded_index in range(orig, local * world):
            rank, within = divmod(padded_index, local)
            rows.append(rank * chunk + offset + within)
        offset += local
    return sorted(rows)


# ----------------------------------------------------------------- pad rows
def kept_rows(rows: int, drop_rows) -> np.ndarray | None:
    """Ascending kept indices, None when nothing drops; refuses out-of-range
    rows (adapters/usp_pad_exclusion.py:79-126)."""
    if not drop_rows:
        return None
    drop = sorted(set(int(r) for r in drop_rows))
    if drop[-1] >= rows or drop[0] < 0:
        raise OracleRefusal(f"a divisibility pad row at index {drop[-1]} was handed to an "
                            f"attention whose axis carries {rows} rows")
    mask = np.ones(rows, dtype=bool)
    mask[drop] = False
    return np.nonzero(mask)[0].astype(np.int64)


def attend_without_pads(q, k, v, drop_rows, kv_drop_rows, attend):
    """Attend over the real rows and write zeros where pads sat
    (adapters/usp_pad_exclusion.py:112-137)."""
    qi = kept_rows(q.shape[1], drop_rows)
    if kv_drop_rows is drop_rows and k.shape[1] == q.shape[1]:
        ki = qi
    else:
        ki = kept_rows(k.shape[1], kv_drop_rows)
    out = attend(q if qi is None else q[:, qi], k if ki is None else k[:, ki],
                 v if ki is None else v[:, ki])
    if qi is None:
        return out
    full = np.zeros(q.shape, dtype=out.dtype)
    full[:, qi] = out
    return full


# ----------------------------------------------------------------- query-group bias
def validate_query_bias_groups(groups, queries: int, keys: int) -> None:
    """Groups must partition [0, queries) in order; each bias broadcasts as
    (B, H, Q, K) over its group and declares at most `keys` keys
    (adapters/usp_query_bias.py:64-92)."""
    cursor = 0
    for start, end, bias in groups:
        if start != cursor or end < start or end > queries:
            raise OracleRefusal(f"group [{start}, {end}) does not continue the partition of "
                                f"[0, {queries}) at row {cursor}")
        cursor = end
        if bias is None:
            continue
        if bias.ndim != 4 or bias.shape[2] not in (1, end - start):
            raise OracleRefusal(f"a bias shaped {bias.shape} does not broadcast over its group")
        if bias.shape[3] > keys:
            raise OracleRefusal(f"a bias declares {bias.shape[3]} keys over a sequence of {keys}")
    if cursor != queries:
        raise OracleRefusal(f"the groups cover {cursor} of {queries} query rows")


def extend_bias_keys(bias: np.ndarray, keys: int) -> np.ndarray:
    """Zero columns for the keys a bias does not declare
    (adapters/usp_query_bias.py:95-106)."""
    short = keys - bias.shape[3]
    if short <= 0:
        return bias
    return np.concatenate([bias, np.zeros((*bias.shape[:3], short), dtype=bias.dtype)], axis=3)


def query_group_attention(q, k, v, groups, scale=None):
    """Each query group attends the whole key axis under its own additive
    bias, float64 (adapters/usp_query_bias.py:109-130); (B, L, H, D) in/out."""
    validate_query_bias_groups(groups, q.shape[1], k.shape[1])
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    qh, kh, vh = (np.asarray(t, dtype=np.float64).transpose(0, 2, 1, 3) for t in (q, k, v))
    out = np.empty_like(qh)
    for start, end, bias in groups:
        if end == start:
            continue
        logits = qh[:, :, start:end] @ kh.transpose(0, 1, 3, 2) * scale
        if bias is not None:
            logits = logits + extend_bias_keys(np.asarray(bias, dtype=np.float64), kh.shape[2])
        logits = logits - logits.max(axis=-1, keepdims=True)
        w = np.exp(logits)
        out[:, :, start:end] = (w / w.sum(axis=-1, keepdims=True)) @ vh
    return out.transpose(0, 2, 1, 3)


def assert_pads_are_a_tail(drop_rows, rows: int) -> None:
    """A biased stream's pad rows must be the sequence tail, or the group
    boundaries would slide (adapters/usp_pad_exclusion.py:129-149)."""
    if drop_rows and list(drop_rows) != list(range(rows - len(drop_rows), rows)):
        raise OracleRefusal(f"a query-group bias met {len(drop_rows)} divisibility pad row(s) "
                            f"away from the tail of its {rows}-row sequence")


def attend_groups_without_pads(q, k, v, drop_rows, kv_drop_rows, groups):
    """The pad exclusion with query-bias groups: tail check, drop, grouped
    attention, zero-restore (adapters/usp_pad_exclusion.py:112-137 with
    groups, adapters/usp_full_axis.py:14-16)."""
    if groups:
        assert_pads_are_a_tail(drop_rows, q.shape[1])
    return attend_without_pads(q, k, v, drop_rows, kv_drop_rows,
                               lambda qq, kk, vv: query_group_attention(qq, kk, vv, groups))


# ----------------------------------------------------------------- NVFP4 activation scale
def round_to_bf16(x) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even), returned as fp32 values; NaN kept."""
    f = np.asarray(x, dtype=np.float32)
    bits = f.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(f), f, out)


def _to_dtype(x, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return round_to_bf16(x)
    if dtype == "float16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(x, dtype=np.float32)


def shared_activation_scale(shards: list[np.ndarray], divisor: float, dtype: str) -> float:
    """The scale one GPU takes over the whole tensor, from its shards: the max
    over shards of amax|x| (fp32), cast to the activation dtype, divided by
    `divisor` in that dtype (adapters/quant_activation_scale.py:222-246)."""
    amax = np.float32(max((float(np.max(np.abs(s))) if s.size else 0.0) for s in shards))
    cast = _to_dtype(amax, dtype)
    return float(_to_dtype(np.float32(cast) / np.float32(divisor), dtype))


def cfg_combine(cond: np.ndarray, uncond: np.ndarray, cfg: float, dtype: str) -> np.ndarray:
    """uncond + (cond - uncond) * cfg with each operation rounded to the
    prediction dtype and the scale taken as fp32: the default combine the
    dual-model CFG split runs after its all-gather
    (actor/dual_model_cfg.py:84-92)."""
    c = _to_dtype(np.asarray(cond, dtype=np.float32), dtype)
    u = _to_dtype(np.asarray(uncond, dtype=np.float32), dtype)
    d = _to_dtype(c - u, dtype)
    m = _to_dtype(d * np.float32(cfg), dtype)
    return _to_dtype(u + m, dtype)


# ----------------------------------------------------------------- joint order
@dataclass(frozen=True)
class RankMajorJointOrder:
    """[t0,i0,t1,i1,...] <-> [t0,t1,...,i0,i1,...] on the gathered axis
    (adapters/usp_sequence_order.py:33-146)."""

    text_rows: int
    image_rows: int

    def world(self, rows: int) -> int:
        local = self.text_rows + self.image_rows
        if self.text_rows < 1 or self.image_rows < 1 or rows % local:
            raise OracleRefusal("the gathered sequence does not tile its local text/image pair")
        world = rows // local
        if world < 2:
            raise OracleRefusal("the Ulysses degree is less than two")
        return world

    def permutation(self, rows: int) -> np.ndarray:
        """canonical index -> rank-major index (usp_sequence_order.py:69-78)."""
        local = self.text_rows + self.image_rows
        starts = np.arange(self.world(rows))[:, None] * local
        text = starts + np.arange(self.text_rows)[None, :]
        image = starts + self.text_rows + np.arange(self.image_rows)[None, :]
        return np.concatenate([text.reshape(-1), image.reshape(-1)]).astype(np.int64)

    @staticmethod
    def inverse(perm: np.ndarray) -> np.ndarray:
        inv = np.empty_like(perm)
        inv[perm] = np.arange(perm.size)
        return inv

    def canonicalize(self, q, k, v, drop_rows, kv_drop_rows):
        """Reorder to stock order and remap pad rows (usp_sequence_order.py:105-146)."""
        if q.shape != k.shape or q.shape != v.shape:
            raise OracleRefusal("q/k/v are not equal B,L,H,D self-attention tensors")
        rows = q.shape[1]
        perm = self.permutation(rows)
        inv = self.inverse(perm)

        def remap(rs):
            if rs is None:
                return None
            for r in rs:
                if r < 0 or r >= rows:
                    raise OracleRefusal("a rank-major pad row is outside the gathered sequence")
            return sorted(int(inv[r]) for r in rs)

        qrows = remap(drop_rows)
        krows = qrows if kv_drop_rows is drop_rows else remap(kv_drop_rows)
        return q[:, perm], k[:, perm], v[:, perm], qrows, krows, perm

    def restore(self, out, perm):
        """Back to rank-major order (usp_sequence_order.py:311-322)."""
        return out[:, self.inverse(perm)]


# ----------------------------------------------------------------- all-to-all
def seq_all_to_all_4d(per_rank: list[np.ndarray], scatter_dim: int, gather_dim: int) -> list[np.ndarray]:
    """yunchang SeqAllToAll4D over a group of len(per_rank) ranks.

    (2, 1): each rank holds (B, S/P, H, D); rank r receives head slice
    [r*H/P, (r+1)*H/P) from every source, concatenated rank-major along the
    sequence -> (B, S, H/P, D).  (1, 2): the inverse -- rank r receives its
    own sequence chunk [r*S/P, (r+1)*S/P) of every source's heads, source
    order along the head axis -> (B, S/P, H, D).  The argument convention and
    the rank-major gathered order are the ones the reference pins
    (adapters/usp_full_axis.py:27-29,40; tests/test_usp_full_axis.py:12-27;
    tests/test_flux_pad_exclusion.py:188-199).
    """
    world = len(per_rank)
    if (scatter_dim, gather_dim) == (2, 1):
        heads = per_rank[0].shape[2]
        if heads % world:
            raise OracleRefusal(f"{heads} heads do not divide the Ulysses degree {world}")
        hl = heads // world
        return [np.concatenate([src[:, :, r * hl:(r + 1) * hl] for src in per_rank], axis=1)
                for r in range(world)]
    if (scatter_dim, gather_dim) == (1, 2):
        rows = per_rank[0].shape[1]
        if rows % world:
            raise OracleRefusal(f"{rows} rows do not divide the Ulysses degree {world}")
        sl = rows // world
        return [np.concatenate([src[:, r * sl:(r + 1) * sl] for src in per_rank], axis=2)
                for r in range(world)]
    raise OracleRefusal(f"unsupported all-to-all ({scatter_dim}, {gather_dim})")


# ----------------------------------------------------------------- attention
def attention_lse(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                  scale: float | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Non-causal softmax(scale q k^T) v and natural-log LSE in float64.

    (B, Lq, H, D) x (B, Lk, Hkv, D) -> out (B, Lq, H, D), lse (B, H, Lq): the
    block-processor contract of adapters/cudnn_ring_attention.py:61-89, with
    the math of its known-answer probe (:123-128).  Grouped K/V heads repeat
    as adapters/base.py:280-292 does (repeat_interleave).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    d = q.shape[-1]
    scale = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    rep = q.shape[2] // k.shape[2]
    if rep > 1:
        k = np.repeat(k, rep, axis=2)
        v = np.repeat(v, rep, axis=2)
    logits = np.einsum("blhd,bmhd->bhlm", q, k) * scale
    mx = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - mx)
    s = e.sum(axis=-1, keepdims=True)
    out = np.einsum("bhlm,bmhd->blhd", e / s, v)
    lse = (mx + np.log(s))[..., 0]
    return out, lse


def lse_merge(outs: list[np.ndarray], lses: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
    """Exact combine of attention over disjoint key blocks (the ring merge the
    reference reaches through adapters/base.py:320)."""
    lse_stack = np.stack([np.asarray(l, dtype=np.float64) for l in lses])  # n B H L
    mx = lse_stack.max(axis=0)
    w = np.exp(lse_stack - mx)
    total = w.sum(axis=0)
    lse = mx + np.log(total)
    out = np.zeros(np.asarray(outs[0]).shape, dtype=np.float64)
    for i, o in enumerate(outs):
        wi = (w[i] / total).transpose(0, 2, 1)[..., None]  # B L H 1
        out += wi * np.asarray(o, dtype=np.float64)
    return out, lse


def ring_attention(q_local: list[np.ndarray], k_local: list[np.ndarray], v_local: list[np.ndarray],
                   scale: float | None = None) -> list[tuple[np.ndarray, np.ndarray]]:
    """Ring attention over R ranks: rank r attends its queries to the key
    block of rank (r - t) mod R at step t, then merges by LSE."""
    world = len(q_local)
    results = []
    for r in range(world):
        parts = [attention_lse(q_local[r], k_local[(r - t) % world], v_local[(r - t) % world], scale)
                 for t in range(world)]
        results.append(lse_merge([p[0] for p in parts], [p[1] for p in parts]))
    return results


def full_context_gather(blocks: list[np.ndarray]) -> np.ndarray:
    """Every rank's (B, L, H, D) block in rank-major slots [r*L, (r+1)*L) of the
    gathered axis (adapters/wan_ring_full_context.py:238-251)."""
    return np.concatenate(blocks, axis=1)


def full_context_ring_attention(q_local, k_local, v_local, scale=None):
    """Local Q of each rank against the gathered K/V in one softmax, no merge
    (adapters/wan_ring_full_context.py:422-449)."""
    k_full, v_full = full_context_gather(k_local), full_context_gather(v_local)
    return [attention_lse(q, k_full, v_full, scale) for q in q_local]


def ulysses_attention(q_local, k_local, v_local, scale=None):
    """Pure Ulysses: head scatter, full-axis attention, inverse all-to-all
    (adapters/usp_full_axis.py:27-40 at ring world 1)."""
    qs = seq_all_to_all_4d(q_local, 2, 1)
    ks = seq_all_to_all_4d(k_local, 2, 1)
    vs = seq_all_to_all_4d(v_local, 2, 1)
    outs = [attention_lse(q, k, v, scale)[0] for q, k, v in zip(qs, ks, vs)]
    return seq_all_to_all_4d(outs, 1, 2)


def hybrid_groups(world: int, ulysses: int, ring: int) -> tuple[list[list[int]], list[list[int]]]:
    """Ulysses and ring groups of a ulysses x ring sequence-parallel world.

    Restates yunchang's set_seq_parallel_pg with use_ulysses_low=True, the
    layout xfuser's initialize_model_parallel hands it
    (actor/worker_env.py:320-327): Ulysses groups are runs of consecutive
    ranks, ring groups stride by the Ulysses degree.  NOT pinned by any
    reference test (the reference stubs xfuser); documented as an assumption.
    """
    sp = ulysses * ring
    if world % sp:
        raise OracleRefusal(f"world {world} is not a multiple of ulysses*ring={sp}")
    uly, rng = [], []
    for dp in range(world // sp):
        off = dp * sp
        for i in range(ring):
            uly.append(list(range(off + i * ulysses, off + (i + 1) * ulysses)))
        for i in range(ulysses):
            rng.append(list(range(off + i, off + sp, ulysses)))
    return uly, rng


# ----------------------------------------------------------------- CFG split
def cfg_take_slice(value, batch: int, world: int, rank: int):
    """This rank's rows of every array whose dim 0 equals the call batch;
    containers recurse (adapters/cfg_parallel.py:71-87)."""
    if isinstance(value, np.ndarray):
        if value.ndim > 0 and value.shape[0] == batch:
            rows = batch // world
            return value[rank * rows:(rank + 1) * rows]
        return value
    if isinstance(value, dict):
        return {k: cfg_take_slice(v, batch, world, rank) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        out = [cfg_take_slice(v, batch, world, rank) for v in value]
        return tuple(out) if isinstance(value, tuple) else out
    return value


def cfg_all_gather(slices: list[np.ndarray]) -> np.ndarray:
    """Reassemble predictions over the cfg group (adapters/cfg_parallel.py:293-301)."""
    return np.concatenate(slices, axis=0)


def cfg_rank_layout(world: int, sp: int, cfg: int) -> list[dict]:
    """(sp_rank, cfg_rank) of each global rank with sequence parallel fastest,
    then cfg (xfuser's group order as used by actor/worker_env.py:320-327)."""
    if world % (sp * cfg):
        raise OracleRefusal("world is not a multiple of sp*cfg")
    return [{"rank": r, "sp_rank": r % sp, "cfg_rank": (r // sp) % cfg} for r in range(world)]


# ----------------------------------------------------------------- prologue math
def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """x * rsqrt(mean(x^2) + eps) * weight over the last axis (the Q/K norm the
    Wan forward applies before the seam, adapters/wan_family.py:70-71)."""
    x = np.asarray(x, dtype=np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * np.asarray(weight, np.float64)


def rope_table(positions: np.ndarray, axes_dim: list[int], theta: float = 10000.0) -> np.ndarray:
    """Per-token rotation angles for multi-axis RoPE.

    positions: (L, n_axes) integer coordinates; axis a contributes axes_dim[a]/2
    frequency pairs with omega_i = theta^(-2i/axes_dim[a]).  Returns (L, D/2)
    angles, pairs of all axes concatenated in axis order (the standard N-D
    rotary embedding; the frequency layout is a parameter of the kernel).
    """
    cols = []
    for a, dim in enumerate(axes_dim):
        omega = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float64) / dim))
        cols.append(positions[:, a:a + 1].astype(np.float64) * omega[None, :])
    return np.concatenate(cols, axis=1)


def apply_rope(x: np.ndarray, angles: np.ndarray) -> np.ndarray:
    """Rotate consecutive pairs (x[2i], x[2i+1]) by angles[l, i]:
    (x0 cos - x1 sin, x0 sin + x1 cos).  x: (B, L, H, D), angles: (L, D/2)."""
    x = np.asarray(x, dtype=np.float64)
    c = np.cos(angles)[None, :, None, :]
    s = np.sin(angles)[None, :, None, :]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out
