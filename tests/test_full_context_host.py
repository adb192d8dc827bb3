"""The Wan Ring2 full-context function's refusals, on the CPU, against the
reference's own verdicts (adapters/wan_ring_full_context.py:17-117) recorded
in tests/golden/ by make_golden.py section (l): every kernel option and local
shard case is accepted or refused exactly as the reference does, with the
reference's message, fp16 and bf16 shards alike."""
from __future__ import annotations

import json
import math
from pathlib import Path

import pytest
import torch

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "golden.json").read_text())


def _decode(x):
    if isinstance(x, dict):
        if set(x) == {"tuple"}:
            return tuple(_decode(y) for y in x["tuple"])
        if set(x) == {"list"}:
            return [_decode(y) for y in x["list"]]
        if set(x) == {"float"}:
            return float(x["float"])
    return x


def _verdict(fn, **kwargs):
    from dgx_monarch_b200.usp import UnsupportedModelError

    try:
        fn(**kwargs)
        return "ok"
    except UnsupportedModelError as exc:
        return str(exc)


@pytest.mark.parametrize("entry", GOLDEN["full_context_surface"], ids=lambda e: str(len(e["verdict"])))
def test_kernel_options_are_judged_as_the_reference_judges_them(entry):
    from dgx_monarch_b200.full_context import validate_flash_surface

    case = {key: _decode(value) for key, value in entry["case"].items()}
    assert _verdict(validate_flash_surface, **case) == entry["verdict"]


@pytest.mark.parametrize("entry", GOLDEN["full_context_qkv"], ids=lambda e: e["case"]["dtype"])
def test_local_shards_are_judged_as_the_reference_judges_them(entry):
    from dgx_monarch_b200.full_context import validate_local_qkv

    case = entry["case"]
    dt = getattr(torch, case["dtype"])
    q, k, v = (torch.zeros(case[n], dtype=dt) for n in "qkv")
    if case.get("grad"):
        q.requires_grad_(True)
    assert _verdict(validate_local_qkv, q=q, k=k, v=v) == entry["verdict"]


def test_the_cases_cover_every_refusal():
    verdicts = {e["verdict"] for e in GOLDEN["full_context_surface"] + GOLDEN["full_context_qkv"]}
    assert "ok" in verdicts
    assert len(verdicts) >= 13
    assert any(math.isinf(_decode(v)) for e in GOLDEN["full_context_surface"]
               for v in e["case"].values() if isinstance(v, dict) and "float" in v)
