"""The FMA-pipe exponential of the tcgen05 attention softmax (ex2_poly in csrc/attention_tc.cu).

A quarter of the softmax exponentials are evaluated as a polynomial instead of on the SFU. This
test reads the polynomial's coefficients from the kernel source and replays the device algorithm
step by step in float32 (clamp at -125, round-to-nearest split with the 1.5 * 2^23 magic number,
degree-4 Horner, exponent-field add), then checks it against float64 2^t:
  * relative error <= 5e-6 for t in [-125, 8] (the softmax exponents are <= 8);
  * every result finite and non-negative, masked scores (t = -inf) at most 2^-125.
"""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SOURCE = Path(__file__).resolve().parents[1] / "attention-rank_b200" / "csrc" / "attention_tc.cu"


def _coefficients() -> list[np.float32]:
    text = SOURCE.read_text()
    body = text[text.index("float ex2_poly(float t)"):]
    body = body[:body.index("\n}\n")]
    numbers = [float(v) for v in re.findall(r"fmaf\([^;]*?(-?\d+\.\d+(?:e-?\d+)?)f\)", body)]
    first = re.search(r"fmaf\((-?\d+\.\d+(?:e-?\d+)?)f, f, (-?\d+\.\d+(?:e-?\d+)?)f\)", body)
    assert first is not None and len(numbers) == 4
    c4, c3 = float(first.group(1)), float(first.group(2))
    c2, c1, c0 = numbers[1], numbers[2], numbers[3]
    return [np.float32(v) for v in (c0, c1, c2, c3, c4)]


def ex2_poly(t: np.ndarray) -> np.ndarray:
    c0, c1, c2, c3, c4 = _coefficients()
    magic = np.float32(12582912.0)
    t = np.maximum(t.astype(np.float32), np.float32(-125.0))
    j = (t + magic).astype(np.float32)
    f = (t - (j - magic).astype(np.float32)).astype(np.float32)
    p = (c4 * f + c3).astype(np.float32)
    p = (p * f + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    bits = (p.view(np.uint32) + (j.view(np.uint32) << np.uint32(23))).astype(np.uint32)
    return bits.view(np.float32)


def test_polynomial_exp2_relative_error():
    t = np.linspace(-125.0, 8.0, 4_000_001, dtype=np.float32)
    got = ex2_poly(t).astype(np.float64)
    want = np.exp2(t.astype(np.float64))
    assert np.max(np.abs(got - want) / want) <= 5e-6


def test_polynomial_exp2_masked_and_underflow():
    t = np.array([-np.inf, -1e30, -300.0, -126.0, -125.5], dtype=np.float32)
    got = ex2_poly(t)
    assert np.all(np.isfinite(got)) and np.all(got >= 0)
    assert np.all(got <= np.float32(2.0 ** -124))
