"""The quantize kernel's rounding rule for 16-bit inputs with fp16 scales, checked in numpy.

The kernel (``pair_codes2`` in ``csrc/sc_quantize.cu``) makes each int8 code without a
division or a tie test: with ``rcp = RN(1/s)``, ``lo = RN(rcp * (1 - 2^-22))`` and
``hi = RN(rcp * (1 + 2^-22))`` it forms ``t1 = RN(x*lo + 1.5*2^23)`` and
``t2 = RN(x*hi + 1.5*2^23)`` (one fma each, exact product) and takes the low byte of
``RN(t1 + t2)``.  These tests replay that arithmetic in numpy (float64 holds the exact
products: 11 + 24 bits) against the reference's rule, ``rint_even(fp32(x) / fp32(s))``
(``speccache/kernels/reference.py:203-204``), for every finite fp16 and bf16 input with
|x| <= 127.5 s over a spread of fp16 scales.  The whole fp16 x fp16 space (1.4e9 pairs) was
checked the same way; a wider bracket (2^-12) fails, which shows the check can fail.
"""

from __future__ import annotations

import numpy as np
import pytest

F32 = np.float32
K_ROUND = np.float64(12582912.0)  # 1.5 * 2^23


def _inputs(kind: str) -> np.ndarray:
    if kind == "f16":
        mags = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float32)
    else:
        mags = (np.arange(0, 0x7F80, dtype=np.uint32) << 16).view(np.float32)
    return np.concatenate([mags, -mags[1:]])


def _rule_codes(x: np.ndarray, s: np.float32, bracket: float) -> np.ndarray:
    rcp = F32(1.0) / s
    lo, hi = F32(rcp * F32(1.0 - bracket)), F32(rcp * F32(1.0 + bracket))
    x64 = x.astype(np.float64)
    t1 = (np.rint(x64 * np.float64(lo)) + K_ROUND).astype(np.float32)
    t2 = (np.rint(x64 * np.float64(hi)) + K_ROUND).astype(np.float32)
    return ((t1 + t2).view(np.uint32) & 0xFF).astype(np.uint8).view(np.int8)


def _reference_codes(x: np.ndarray, s: np.float32) -> np.ndarray:
    return np.rint((x / s).astype(np.float64)).astype(np.int64).astype(np.int8)


def _mismatches(kind: str, bracket: float, step: int) -> int:
    xs = _inputs(kind)
    scales = np.arange(1, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float32)
    bad = 0
    for s in scales[::step]:
        x = xs[np.abs(xs) <= F32(127.5) * s]
        bad += int(np.count_nonzero(_rule_codes(x, s, bracket) != _reference_codes(x, s)))
    return bad


@pytest.mark.parametrize("kind", ["f16", "bf16"])
def test_two_product_rule_matches_ieee_division(kind):
    assert _mismatches(kind, 2.0**-22, step=97) == 0


def test_a_wide_bracket_is_caught():
    assert _mismatches("f16", 2.0**-12, step=97) > 0


def test_exact_ties_round_half_even():
    # s = 3/64 has an inexact reciprocal; (k + 1/2) s are exact half-integer quotients
    s = F32(3.0 / 64.0)
    k = np.arange(-127, 127, dtype=np.float32)
    x = ((k + F32(0.5)) * s).astype(np.float16).astype(np.float32)
    assert np.array_equal(x / s, k + F32(0.5))
    codes = _rule_codes(x, s, 2.0**-22).astype(np.int64)
    assert np.array_equal(codes, np.rint(k + 0.5).astype(np.int64))
    assert np.all(codes % 2 == 0)
