"""The one-correction quotient used for softmax weights, checked on the CPU.

``quot_nr(x, T, r)`` with r = rn(1 / T): q = rn(x r), e = x - q T (exact with
an FMA), q1 = rn(q + e r).  The weights' error budget needs q1 within one ulp
of x / T.  float32 steps are emulated exactly with Python fractions.
"""
from fractions import Fraction

import numpy as np

F32 = np.float32


def rn32(v: Fraction) -> np.float32:
    """Round an exact rational to the nearest fp32 (ties to even)."""
    f = F32(float(v))                      # float(): nearest double
    # correct a possible double rounding by checking the neighbours exactly
    best = f
    for cand in (np.nextafter(f, F32(np.inf), dtype=np.float32), np.nextafter(f, F32(-np.inf), dtype=np.float32)):
        if abs(Fraction(float(cand)) - v) < abs(Fraction(float(best)) - v):
            best = cand
    return best


def quot_nr(x: np.float32, T: np.float32, r: np.float32) -> np.float32:
    q = rn32(Fraction(float(x)) * Fraction(float(r)))
    e = rn32(-Fraction(float(q)) * Fraction(float(T)) + Fraction(float(x)))
    return rn32(Fraction(float(e)) * Fraction(float(r)) + Fraction(float(q)))


def ulp(v: np.float32) -> float:
    return float(np.spacing(np.abs(v)))


def test_one_correction_quotient_within_one_ulp():
    rng = np.random.default_rng(7)
    xs = np.concatenate([rng.normal(0, 3, 1500), rng.uniform(-60, 60, 500)]).astype(np.float32)
    Ts = np.concatenate([rng.uniform(0.05, 3.0, 1500), [0.7, 1.3, 0.1, 3.0, 7.0] * 100]).astype(np.float32)
    worst = 0.0
    for x, T in zip(xs, Ts):
        r = rn32(1 / Fraction(float(T)))
        q1 = quot_nr(x, T, r)
        exact = Fraction(float(x)) / Fraction(float(T))
        err = abs(Fraction(float(q1)) - exact)
        if x != 0:
            worst = max(worst, float(err) / ulp(rn32(exact)))
        assert err <= Fraction(ulp(rn32(exact))), (x, T, q1)
    assert worst < 1.0


def test_split_log2e_product():
    """exp(d) = 2^(d log2 e) with the product kept as hi + lo (log2 e split
    into fp32 L1 + L2): hi + lo must equal d log2 e to about 2^-40 relative,
    leaving the hardware 2^x approximation as the only sizeable error."""
    import math
    L1 = np.float32(1.4426950216293335)
    L2 = np.float32(1.925963033500011e-08)
    log2e = Fraction(1) / Fraction(math.log(2))          # float64-accurate log2(e)
    assert abs(Fraction(float(L1)) + Fraction(float(L2)) - log2e) < Fraction(1, 2 ** 49)
    rng = np.random.default_rng(11)
    for d in -np.abs(rng.normal(0, 20, 3000)).astype(np.float32):
        hi = rn32(Fraction(float(d)) * Fraction(float(L1)))
        inner = rn32(Fraction(float(d)) * Fraction(float(L1)) - Fraction(float(hi)))   # fmaf(d, L1, -hi)
        lo = rn32(Fraction(float(d)) * Fraction(float(L2)) + Fraction(float(inner)))    # fmaf(d, L2, inner)
        exact = Fraction(float(d)) * log2e
        err = abs(Fraction(float(hi)) + Fraction(float(lo)) - exact)
        assert err <= abs(exact) * Fraction(1, 2 ** 40) + Fraction(1, 2 ** 60), (d, float(err))
