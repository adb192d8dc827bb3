"""The ring block processor on the GPU: the reference's two admission checks
(the dyadic known-answer probe of adapters/cudnn_ring_attention.py:106-135
and the capability probe of adapters/attention_capability.py:151-211) pass,
the recorded probe tensors give the recorded (out, lse), and four ring blocks
through the processor merge into attention over every key."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.test_attn_gpu import BF16_REL_L2, LSE_ABS, reference_attention, rel_l2

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_dyadic_probe_passes(lib):
    from dgx_monarch_b200.ring_processor import B200RingBlockProcessor, probe_dyadic

    probe_dyadic(B200RingBlockProcessor())


def test_recorded_probe_tensors_give_the_recorded_results(lib):
    from dgx_monarch_b200.ring_processor import B200RingBlockProcessor

    spec = json.loads((GOLDEN / "golden.json").read_text())["probe"]
    arr = np.load(GOLDEN / "golden_arrays.npz")
    proc = B200RingBlockProcessor()
    assert {c["dtype"] for c in spec} == {"torch.float16", "torch.bfloat16"}
    for case in spec:
        dt = torch.float16 if "float16" in case["dtype"] and "bfloat16" not in case["dtype"] else torch.bfloat16
        q, k, v = (torch.from_numpy(arr[f"probe_{case['index']}_{n}"]).cuda().to(dt) for n in "qkv")
        out, lse = proc(q, k, v, softmax_scale=case["scale"])
        want_out = torch.from_numpy(arr[f"probe_{case['index']}_out"]).cuda()
        want_lse = torch.from_numpy(arr[f"probe_{case['index']}_lse"]).cuda()
        eps = torch.finfo(dt).eps
        assert out.dtype == dt and lse.dtype == torch.float32 and lse.shape == want_lse.shape
        assert torch.allclose(lse, want_lse, atol=2e-5, rtol=2e-5)
        assert torch.allclose(out.float(), want_out, atol=eps / 8, rtol=2 * eps)


@pytest.mark.parametrize("head_dim", [64, 96, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_capability_probe_admits_the_kernel(lib, head_dim, dtype):
    from types import SimpleNamespace

    from dgx_monarch_b200.ring_processor import B200RingBlockProcessor, assert_kernel_capability

    assert_kernel_capability("Flux", head_dim, SimpleNamespace(manual_cast_dtype=dtype))
    zeros = torch.zeros(1, 128, 2, head_dim, device="cuda", dtype=dtype)
    out, lse = B200RingBlockProcessor()(zeros, zeros, zeros)
    assert torch.equal(out, torch.zeros_like(out))
    assert torch.allclose(lse, torch.full_like(lse, float(np.log(128))), atol=1e-5)


def test_capability_probe_refuses_a_model_the_kernel_cannot_run(lib):
    from types import SimpleNamespace

    from dgx_monarch_b200.ring_processor import assert_kernel_capability
    from dgx_monarch_b200.usp import UnsupportedModelError

    with pytest.raises(UnsupportedModelError, match=r"declined a probe.*float32.*UnsupportedModelError"):
        assert_kernel_capability("Fp32Family", 128, SimpleNamespace(manual_cast_dtype=torch.float32))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_ring_blocks_through_the_processor_merge_to_full_attention(lib, dtype):
    """xfuser's ring calls the processor once per key/value block and merges
    by the returned fp32 LSE; four blocks of one rank's view, merged, equal
    attention over the whole key axis."""
    from dgx_monarch_b200.ops import lse_merge
    from dgx_monarch_b200.ring_processor import B200RingBlockProcessor

    g = torch.Generator(device="cuda").manual_seed(12)
    q = torch.randn(2, 500, 3, 128, device="cuda", generator=g).to(dtype)
    k, v = (torch.randn(2, 4 * 300, 3, 128, device="cuda", generator=g).to(dtype) for _ in range(2))
    proc = B200RingBlockProcessor()
    parts = [proc(q, k[:, i * 300:(i + 1) * 300], v[:, i * 300:(i + 1) * 300], softmax_scale=None)
             for i in range(4)]
    out, lse = lse_merge([p[0].contiguous() for p in parts], [p[1] for p in parts], out_dtype=dtype)
    ref, ref_lse = reference_attention(q, k, v)
    assert rel_l2(out, ref) <= BF16_REL_L2
    assert (lse - ref_lse).abs().max().item() <= LSE_ABS


def test_non_positive_scale_is_refused_on_device_tensors(lib):
    from dgx_monarch_b200.ring_processor import B200RingBlockProcessor
    from dgx_monarch_b200.usp import UnsupportedModelError

    x = torch.zeros(1, 8, 2, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(UnsupportedModelError, match="positive scale"):
        B200RingBlockProcessor()(x, x, x, softmax_scale=0.0)
