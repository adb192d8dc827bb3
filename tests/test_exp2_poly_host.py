"""The polynomial 2^x of the attention kernel's softmax (exp2_poly2 in
csrc/ptx.cuh), emulated step by step in float32 on the CPU with the
coefficients read from that source: Cody-Waite range reduction with the
1.5 * 2^23 rounding constant, the degree-3 polynomial, the exponent added in
the integer domain, and the clamp at -125.  The relative error stays within
the 7.5e-5 the source states, far below the bf16 rounding of P."""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "dgx_monarch_b200" / "csrc" / "ptx.cuh"


def _coefficients() -> list[float]:
    text = SRC.read_text()
    body = text[text.index("uint64_t exp2_poly2"):]
    body = body[:body.index("\n}\n")]
    found = [float(x) for x in re.findall(r"pk2\(([-0-9.e]+)f, \1f\)", body)]
    return [c for c in found if c > 0]  # the polynomial's; -1 belongs to the range reduction


def _fma(a, b, c):
    """fp32 fused multiply-add: one rounding of the exact a * b + c."""
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def _exp2_poly(x: np.ndarray) -> np.ndarray:
    magic = np.float32(12582912.0)
    c3, c2, c1, c0 = (np.float32(c) for c in _coefficients())
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    t = (x + magic).astype(np.float32)
    jf = (t - magic).astype(np.float32)
    f = _fma(jf, np.float32(-1.0), x)
    p = _fma(f, c3, c2)
    p = _fma(p, f, c1)
    p = _fma(p, f, c0)
    bits = p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def test_source_holds_the_rounding_constant_and_four_coefficients():
    body = SRC.read_text()
    assert re.search(r"kMagic = 12582912\.0f", body)
    coef = _coefficients()
    assert len(coef) == 4 and all(0 < c < 1.1 for c in coef)


def test_relative_error_within_the_stated_bound():
    x = np.concatenate([np.linspace(-124.0, 0.0, 400001, dtype=np.float32),
                        np.float32(-np.arange(0, 124, 1.0 / 64))])
    got = _exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() <= 7.5e-5 * 1.01, rel.max()


def test_inputs_below_the_clamp_stay_normal_and_tiny():
    got = _exp2_poly(np.array([-125.0, -200.0, -1e30], dtype=np.float32))
    assert np.all(got > 0) and np.all(got <= np.float32(2.0 ** -124))
    assert np.all(np.isfinite(got))
