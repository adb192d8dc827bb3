"""The Wan Ring2 full-context ring function, on the B200 kernels.

The reference installs `full_context_ring_attention` as xfuser's
`ring_attn_fn` for pure ring-2 Wan renders
(adapters/wan_ring_full_context.py:298-449, bound at
adapters/wan_ring_attention.py:360-451): each batch item's K/V is gathered
into sequence-rank slots, then one ATen flash call attends the local query
rows against the full key axis, which avoids the bf16-LSE ring merge.

`make_full_context_ring_attention` returns a function with that signature and
those refusals.  Inside, one kernel stores every batch item's K/V block into
rank-major slots of every rank's peer window (NVLink), a flag barrier
follows, and one attention kernel reads the gathered axis in place
(`dgxm_full_context_attn_fwd`).  Every refusal is raised before any
communication, on every rank alike, as the reference's validators are.
"""
from __future__ import annotations

import math

import torch

from .ring import FullContextRingAttention
from .usp import UnsupportedModelError

_SUPPORTED = (torch.float16, torch.bfloat16)


def validate_flash_surface(*, dropout_p, softmax_scale, causal, window_size, softcap,
                           alibi_slopes, return_softmax) -> None:
    """The kernel options the full-context call takes: dropout 0, a finite
    positive scale, non-causal, no window, no softcap, no ALiBi, no returned
    probabilities (adapters/wan_ring_full_context.py:63-117)."""
    def number(x):
        return not isinstance(x, bool) and isinstance(x, (int, float)) and math.isfinite(float(x))

    if not number(dropout_p) or float(dropout_p) != 0.0:
        raise UnsupportedModelError("Wan ring TORCH_FLASH supports dropout_p=0 only")
    if softmax_scale is not None and (not number(softmax_scale) or float(softmax_scale) <= 0.0):
        raise UnsupportedModelError("Wan ring TORCH_FLASH requires a finite positive softmax scale")
    if causal is not False:
        raise UnsupportedModelError("Wan ring TORCH_FLASH supports non-causal attention only")
    if (type(window_size) is not tuple or len(window_size) != 2
            or any(isinstance(x, bool) or not isinstance(x, int) for x in window_size)
            or window_size != (-1, -1)):
        raise UnsupportedModelError("Wan ring TORCH_FLASH does not support local attention windows")
    if not number(softcap) or float(softcap) != 0.0:
        raise UnsupportedModelError("Wan ring TORCH_FLASH does not support softcap")
    if alibi_slopes is not None:
        raise UnsupportedModelError("Wan ring TORCH_FLASH does not support ALiBi")
    if return_softmax is not False:
        raise UnsupportedModelError(
            "Wan ring TORCH_FLASH does not support returning attention probabilities")


def validate_local_qkv(q, k, v) -> None:
    """Equal local (B, L, H, 128) fp16 or bf16 shards on one CUDA device,
    inference only (adapters/wan_ring_full_context.py:17-60)."""
    if any(not isinstance(t, torch.Tensor) for t in (q, k, v)):
        raise UnsupportedModelError("Wan ring TORCH_FLASH requires tensor q/k/v inputs")
    if any(t.requires_grad for t in (q, k, v)):
        raise UnsupportedModelError("Wan ring TORCH_FLASH is inference-only")
    if any(t.ndim != 4 for t in (q, k, v)):
        raise UnsupportedModelError("Wan ring TORCH_FLASH requires 4D q/k/v")
    if k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[2:] != k.shape[2:]:
        raise UnsupportedModelError(
            "Wan ring TORCH_FLASH requires equal K/V shapes and matching q/k/v batch, head, and "
            "head-dimension shapes")
    if any(size < 1 for t in (q, k, v) for size in t.shape):
        raise UnsupportedModelError("Wan ring TORCH_FLASH requires non-empty q/k/v")
    if q.dtype not in _SUPPORTED or any(t.dtype != q.dtype for t in (k, v)):
        raise UnsupportedModelError("Wan ring TORCH_FLASH is validated for matching FP16/BF16 q/k/v only")
    if q.shape[-1] != 128:
        raise UnsupportedModelError("Wan ring TORCH_FLASH is validated for head dimension 128 only")
    if q.device.type != "cuda" or any(t.device != q.device for t in (k, v)):
        raise UnsupportedModelError("Wan ring TORCH_FLASH requires q/k/v on one CUDA device")
    if any(t.layout != torch.strided for t in (q, k, v)):
        raise UnsupportedModelError("Wan ring TORCH_FLASH requires strided tensors")
    if q.shape != k.shape:
        raise UnsupportedModelError("Wan ring TORCH_FLASH requires equal local q/k/v shapes")


def make_full_context_ring_attention(*, ring_group, generation: int = 1,
                                     device: torch.device | None = None):
    """`ring_attn_fn` for a pure ring-2 group: local Q x full K/V, exact."""
    import torch.distributed as dist

    if not dist.is_initialized():
        raise UnsupportedModelError("Wan ring full-context distributed authority is unavailable")
    world = dist.get_world_size(ring_group)
    rank = dist.get_rank(ring_group)
    if world != 2:
        raise UnsupportedModelError("Wan ring full-context gather requires ring world 2")
    device = device or torch.device("cuda", torch.cuda.current_device())
    plans: dict = {}

    @torch.compiler.disable
    def full_context_ring_attention(q, k, v, dropout_p=0.0, softmax_scale=None, causal=False,
                                    window_size=(-1, -1), alibi_slopes=None, deterministic=False,
                                    return_attn_probs=False, group=None, attn_type=None,
                                    attn_processor=None, attn_layer=None, joint_tensor_key=None,
                                    joint_tensor_value=None, joint_strategy="none",
                                    q_descale=None, k_descale=None, v_descale=None):
        validate_flash_surface(dropout_p=dropout_p, softmax_scale=softmax_scale, causal=causal,
                               window_size=window_size, softcap=0.0, alibi_slopes=alibi_slopes,
                               return_softmax=return_attn_probs)
        validate_local_qkv(q, k, v)
        if deterministic is not False:
            raise UnsupportedModelError("Wan ring full-context attention requires deterministic=False")
        if (attn_layer is not None or joint_tensor_key is not None or joint_tensor_value is not None
                or joint_strategy != "none" or q_descale is not None or k_descale is not None
                or v_descale is not None):
            raise UnsupportedModelError(
                "Wan ring full-context attention received an unsupported xFuser surface")
        if group is not None and group is not ring_group:
            raise UnsupportedModelError("Wan ring full-context attention received the wrong process group")
        if softmax_scale is not None and float(softmax_scale) != 1.0 / math.sqrt(q.shape[-1]):
            raise UnsupportedModelError("Wan ring TORCH_FLASH requires the default head-dimension scale")
        if plans.get("closed"):
            raise UnsupportedModelError("this full-context ring belongs to a retired setup generation")
        b, l, h, d = q.shape
        key = (b, l, h, k.shape[2], d, q.dtype)
        plan = plans.get(key)
        if plan is None:
            plan = FullContextRingAttention(world=world, rank=rank, batch=b, q_len=l, kv_len=l, heads=h,
                                            kv_heads=k.shape[2], head_dim=d, device=device,
                                            group=ring_group, generation=generation, dtype=q.dtype)
            plans[key] = plan
        out, _ = plan.forward(q, k, v)
        return out

    def invalidate() -> None:
        """Release the windows of this generation (actor/attention_dispatch.py:383-401)."""
        for key, plan in list(plans.items()):
            if key != "closed":
                plan.close()
        plans.clear()
        plans["closed"] = True

    full_context_ring_attention.invalidate = invalidate
    return full_context_ring_attention
