"""The ring block processor and the kernel's capability probes.

xfuser's ring loop (reached from adapters/base.py:320 when the ring degree
exceeds one) calls one block processor per key/value block and merges the
partial results by their log-sum-exp.  The reference carries a cuDNN
processor for this because the stock flash path rounds the block LSE to the
query dtype (adapters/cudnn_ring_attention.py:61-89); `B200RingBlockProcessor`
is the same contract on the tcgen05 kernel: (q, k, v) blocks of (B, L, H, D)
fp16 or bf16 in, the block output in the inputs' dtype and its natural-log
LSE in fp32 (B, H, L) out.  Head dimensions up to 64 run on the head-dim-64
kernel, larger ones below 128 (multiples of 8) zero-padded to 128, with the
scale of their own head dimension.

The reference admits a processor only after two live checks, restated here on
this kernel:
- `probe_dyadic` -- the known-answer probe of
  adapters/cudnn_ring_attention.py:106-135: inputs whose logits are exact in
  fp16 and bf16, so the LSE must be right to 2e-5 and the output to one
  16-bit rounding;
- `assert_kernel_capability` -- the probe of
  adapters/attention_capability.py:151-211: one forward over
  (1, 128, 2, head_dim) zeros in the model's compute dtype with the keywords
  xfuser's ring forward passes, behind the static head-dimension limit of
  the capability table (128 for this kernel).

Refusals carry the reference's class tag ("[dgxm:P] ...", refusal.py), the
reference processor's conditions and sentences with this kernel's name, and
are raised before any device work, on every rank alike.
"""
from __future__ import annotations

import math

import torch

from .usp import UnsupportedModelError

KERNEL_NAME = "B200_SP"
KERNEL_HEAD_DIM = 128           # the largest head dimension; smaller ones run at 64 or 128
HEAD_DIM_LIMIT = {KERNEL_NAME: KERNEL_HEAD_DIM}  # the capability-table entry this kernel adds
PROBE_SHAPE = (1, 128, 2)       # batch, tokens, heads of the capability probe
_DTYPES = (torch.float16, torch.bfloat16)


def tagged(text: str, troubleshooting: int | None = None) -> str:
    """A class-P (physics) refusal in the reference's tagged form."""
    body = text.strip()
    if troubleshooting is not None:
        body = f"{body} See docs/TROUBLESHOOTING.md #{troubleshooting}."
    return f"[dgxm:P] {body}"


def _refuse(text: str) -> UnsupportedModelError:
    return UnsupportedModelError(tagged(text))


def validate_block_call(q, k, v, *, dropout_p, softmax_scale, causal, window_size, softcap,
                        alibi_slopes, return_softmax, deterministic, extra) -> None:
    """The processor contract, checked in the reference's order: the kernel
    options (maskless non-causal inference, no window / ALiBi / softcap, no
    returned probabilities, no determinism request, a finite scale), then the
    blocks (4-D strided non-empty inference tensors, matching batch, heads
    and head dimension, equal K/V lengths, matching fp16 or bf16, one CUDA
    device).  One condition is this kernel's own and comes last: a
    non-positive scale, which the reference's cuDNN call would take."""
    if extra:
        raise _refuse(f"Ring {KERNEL_NAME} received unsupported processor arguments. Use the supported "
                      "maskless inference arguments or run this workflow on a single topology.")
    if dropout_p != 0.0 or causal is not False:
        raise _refuse(f"Ring {KERNEL_NAME} supports non-causal inference attention only. Use non-causal "
                      "inference or run this workflow on a single topology.")
    if window_size != (-1, -1) or alibi_slopes is not None or softcap != 0.0:
        raise _refuse(f"Ring {KERNEL_NAME} does not support window, ALiBi, or softcap. Use unwindowed "
                      "attention without ALiBi or softcap, or run this workflow on a single topology.")
    if return_softmax is not False:
        raise _refuse(f"Ring {KERNEL_NAME} does not return attention probabilities. Use the attention "
                      "output without requesting probability tensors.")
    if deterministic is not False:
        raise _refuse(f"Ring {KERNEL_NAME} cannot honor deterministic attention. Use the supported "
                      "inference mode or run this workflow on a single topology with a deterministic kernel.")
    if softmax_scale is not None:
        finite = (not isinstance(softmax_scale, bool) and isinstance(softmax_scale, (int, float))
                  and math.isfinite(float(softmax_scale)))
        if not finite:
            raise _refuse(f"Ring {KERNEL_NAME} requires a finite scale. Use a finite numeric softmax scale "
                          "or the default scale.")
    blocks = (q, k, v)
    if not all(isinstance(t, torch.Tensor) for t in blocks):
        raise _refuse(f"Ring {KERNEL_NAME} requires tensor Q/K/V. Use tensor query, key and value inputs.")
    if any(t.ndim != 4 or t.layout != torch.strided or t.numel() == 0 or t.requires_grad for t in blocks):
        raise _refuse(f"Ring {KERNEL_NAME} requires nonempty strided inference Q/K/V. Use nonempty strided "
                      "tensors without gradient tracking.")
    same_bhd = all(t.shape[0] == q.shape[0] and t.shape[2:] == q.shape[2:] for t in (k, v))
    if not same_bhd or k.shape[1] != v.shape[1]:
        raise _refuse(f"Ring {KERNEL_NAME} requires matching B/H/D and K/V length. Use matching batch, head "
                      "and feature dimensions, with equal key/value sequence lengths.")
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise _refuse(f"Ring {KERNEL_NAME} requires matching fp16 or bf16 Q/K/V. Use matching FP16 or BF16 "
                      "query, key and value tensors.")
    if q.device.type != "cuda" or k.device != q.device or v.device != q.device:
        raise _refuse(f"Ring {KERNEL_NAME} requires Q/K/V on one CUDA device. Use query, key and value "
                      "tensors on the same local CUDA device.")
    if softmax_scale is not None and float(softmax_scale) <= 0.0:
        # The kernel's descriptor reads a non-positive scale as "the default",
        # so one is refused rather than silently replaced.
        raise _refuse(f"Ring {KERNEL_NAME} requires a positive scale. Use a positive softmax scale or the "
                      "default scale.")


class B200RingBlockProcessor:
    """One ring block: (out (B, Lq, H, D) in q's dtype, lse fp32 (B, H, Lq))."""

    __slots__ = ()

    def __call__(self, q, k, v, *, dropout_p=0.0, softmax_scale=None, causal=False,
                 window_size=(-1, -1), softcap=0.0, alibi_slopes=None, return_softmax=False,
                 deterministic=False, **kwargs):
        validate_block_call(q, k, v, dropout_p=dropout_p, softmax_scale=softmax_scale, causal=causal,
                            window_size=window_size, softcap=softcap, alibi_slopes=alibi_slopes,
                            return_softmax=return_softmax, deterministic=deterministic, extra=kwargs)
        head_dim = q.shape[-1]
        if head_dim > KERNEL_HEAD_DIM or head_dim % 8:
            raise _refuse(f"{KERNEL_NAME} carries head dimensions up to {KERNEL_HEAD_DIM} in multiples of "
                          f"8, and this block has {head_dim}. Run this workflow on a cfg or single topology.")
        from .ops import attention_fwd, kernel_head_dim

        scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(head_dim)
        dk = kernel_head_dim(head_dim)
        if head_dim < dk:
            # Zero columns add exact zeros to every logit and give zero output
            # columns, which are dropped.
            pad = (0, dk - head_dim)
            q, k, v = (torch.nn.functional.pad(t, pad) for t in (q, k, v))
        elif any(t.stride(-1) != 1 for t in (q, k, v)):
            q, k, v = (t.contiguous() for t in (q, k, v))
        out, lse = attention_fwd(q, k, v, softmax_scale=scale)
        return out[..., :head_dim], lse


def probe_dyadic(processor, *, device: torch.device | None = None) -> None:
    """The known-answer probe, for fp16 and bf16: two heads of 32 queries
    against 64 keys in two groups whose logits (query position x key
    coordinate, times 1/8) are exact in both formats, values 0.25 / 0.75 and
    -0.5 / 1.0 by group.  The LSE must match exact attention to 2e-5 and the
    output to a sixteenth of the format's epsilon absolute or twice it
    relative; a layout or scaling mistake fails both."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    for dtype in _DTYPES:
        pos = torch.arange(32, dtype=torch.float32, device=device) / 16 - 1
        q = torch.zeros(1, 32, 2, 64, device=device, dtype=dtype)
        q[0, :, 0, 0], q[0, :, 1, 0] = pos, -pos
        k = torch.zeros(1, 64, 2, 64, device=device, dtype=dtype)
        k[0, 32:, 0, 0] = 1
        k[0, :32, 1, 0], k[0, 32:, 1, 0] = 2, -1
        v = torch.zeros_like(k)
        for col, (first, second) in enumerate(((0.25, 0.75), (-0.5, 1.0))):
            v[0, :32, :, col], v[0, 32:, :, col] = first, second
        scale = 1.0 / 8.0
        out, lse = processor(q, k, v, softmax_scale=scale)
        logits = torch.einsum("bqhd,bkhd->bhqk", q.float(), k.float()) * scale
        want_lse = torch.logsumexp(logits, dim=-1)
        want = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(logits, dim=-1), v.float()).to(dtype)
        if not torch.allclose(lse, want_lse, atol=2e-5, rtol=2e-5):
            raise RuntimeError(f"{KERNEL_NAME} ring probe returned an incorrect LSE in {dtype}")
        eps = torch.finfo(dtype).eps
        if out.shape != q.shape or out.dtype != dtype or not torch.allclose(out, want, atol=eps / 8,
                                                                             rtol=2 * eps):
            raise RuntimeError(f"{KERNEL_NAME} ring probe returned an incorrect output in {dtype}")


def compute_dtype(model) -> torch.dtype:
    """The dtype a model attends in: its manual-cast or diffusion-model dtype
    when that is a float of at least 16 bits, else bf16."""
    for value in (getattr(model, "manual_cast_dtype", None),
                  getattr(getattr(model, "diffusion_model", None), "dtype", None)):
        if isinstance(value, torch.dtype) and value.is_floating_point and value.itemsize >= 2:
            return value
    return torch.bfloat16


def assert_kernel_capability(family: str, head_dim: int | None, model=None, *, processor=None,
                             device=None) -> None:
    """Refuse, before any collective, a family this kernel cannot attend: first
    the static limit of 128, then one live forward of the ring block over
    (1, 128, 2, head_dim) zeros in the model's compute dtype with the
    keywords xfuser's ring forward passes.  Every rank reaches the same
    verdict, since every input derives from the declared head dimension and
    the model's dtype."""
    if head_dim is None:
        return
    if head_dim > KERNEL_HEAD_DIM:
        raise UnsupportedModelError(tagged(
            f"{KERNEL_NAME} carries head dimensions up to {KERNEL_HEAD_DIM}, and {family} has {head_dim}, "
            "so the sharded attention this topology installs would abort inside the ring instead of "
            "rendering. Run this workflow on a cfg or single topology instead.", troubleshooting=98))
    processor = processor or B200RingBlockProcessor()
    device = device or torch.device("cuda", torch.cuda.current_device())
    dtype = compute_dtype(model)
    blocks = [torch.zeros(*PROBE_SHAPE, head_dim, dtype=dtype, device=device) for _ in range(3)]
    try:
        processor(*blocks, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1),
                  softcap=0.0, alibi_slopes=None, return_softmax=False)
    except torch.cuda.OutOfMemoryError:
        raise
    except Exception as exc:
        b, n, h = PROBE_SHAPE
        raise UnsupportedModelError(tagged(
            f"{KERNEL_NAME} declined a probe of this render's attention on this hardware. The probe for "
            f"{family} ran {h} heads over {n} tokens at head dimension {head_dim} in {dtype} with no "
            f"mask, and the kernel raised {type(exc).__name__}. Run this workflow on a cfg or single "
            "topology instead.", troubleshooting=98)) from exc
