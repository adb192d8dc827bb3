"""The ring block processor's contract on the CPU: every call the reference's
cuDNN ring processor accepts or refuses (adapters/cudnn_ring_attention.py:
26-89, verdicts recorded in tests/golden/ by make_golden.py section (n)) is
judged the same way here, with the same class-tagged sentence naming this
kernel instead of TORCH_CUDNN; and the capability check's static limit."""
from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "golden.json").read_text())


def _decode(x):
    if isinstance(x, dict):
        if set(x) == {"tuple"}:
            return tuple(_decode(y) for y in x["tuple"])
        if set(x) == {"float"}:
            return float(x["float"])
    return x


@pytest.mark.parametrize("entry", GOLDEN["ring_processor"], ids=lambda e: str(e["case"])[:60])
def test_block_calls_are_judged_as_the_reference_judges_them(entry):
    from dgx_monarch_b200.ring_processor import B200RingBlockProcessor
    from dgx_monarch_b200.usp import UnsupportedModelError

    case = entry["case"]
    dt = getattr(torch, case.get("dtype", "bfloat16"))
    q, k, v = (torch.zeros(case.get(n, [1, 8, 2, 64]), dtype=dt) for n in "qkv")
    if "k_dtype" in case:
        k = k.to(getattr(torch, case["k_dtype"]))
    if case.get("grad"):
        q.requires_grad_(True)
    kwargs = {key: _decode(value) for key, value in case.get("kw", {}).items()}
    try:
        B200RingBlockProcessor()(q, k, v, **kwargs)
        got = "ok"
    except UnsupportedModelError as exc:
        got = str(exc)
    assert got == entry["verdict"].replace("TORCH_CUDNN", "B200_SP")


def test_the_cases_reach_every_refusal():
    verdicts = {e["verdict"].split(".")[0] for e in GOLDEN["ring_processor"]}
    assert len(verdicts) == 10
    assert all(v.startswith("[dgxm:P] Ring TORCH_CUDNN") for v in verdicts)


def test_capability_refuses_heads_beyond_the_table_limit_before_any_device_work():
    from dgx_monarch_b200.ring_processor import HEAD_DIM_LIMIT, assert_kernel_capability
    from dgx_monarch_b200.usp import UnsupportedModelError

    assert HEAD_DIM_LIMIT == {"B200_SP": 128}
    with pytest.raises(UnsupportedModelError, match=r"^\[dgxm:P\] B200_SP carries head dimensions up to 128, "
                                                    r"and Ideogram4 has 256.*#98\.$"):
        assert_kernel_capability("Ideogram4", 256, device=torch.device("cpu"))
    assert_kernel_capability("AnyFamily", None)  # no declared head: nothing to check


def test_compute_dtype_follows_the_model():
    from types import SimpleNamespace

    from dgx_monarch_b200.ring_processor import compute_dtype

    assert compute_dtype(None) == torch.bfloat16
    assert compute_dtype(SimpleNamespace(manual_cast_dtype=torch.float16)) == torch.float16
    assert compute_dtype(SimpleNamespace(manual_cast_dtype=torch.float8_e4m3fn,
                                         diffusion_model=SimpleNamespace(dtype=torch.float32))) == torch.float32
