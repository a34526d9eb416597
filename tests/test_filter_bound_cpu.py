"""The FAST filter's division-free bound, checked numerically on the CPU.

The kernel filters on x before any division by T; a candidate may only be
dropped when rn(x / T) < rn(v / T) for the bound's anchor v.  The exact bound
is the smallest fp32 x with rn(x / T) >= rn(v / T); ``fast_lower_bound`` uses
fmaf(-|v|, 2^-20, v) instead, which must never exceed it (one relative
rounding error of a quotient is at most 2^-24 in the normal range).
"""
import numpy as np

F32 = np.float32


def exact_bound(v: np.float32, T: np.float32) -> np.float32:
    """Smallest fp32 x with rn(x / T) >= rn(v / T) (walk down from v)."""
    ty = F32(v / T)
    x = v
    while True:
        nx = np.nextafter(x, F32(-np.inf), dtype=np.float32)
        if F32(nx / T) >= ty:
            x = nx
        else:
            return x


def fast_bound(v: np.float32) -> np.float32:
    # fmaf(-a, 2^-20, v): the exact value v - a * 2^-20, rounded once to fp32
    return F32(np.float64(v) - np.float64(abs(v)) * 2.0 ** -20)


def test_fast_bound_never_exceeds_exact_bound():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.normal(0, 3, 3000), rng.uniform(-40, 40, 1000),
                           rng.choice([-1, 1], 500) * 2.0 ** rng.uniform(-50, 50, 500)]).astype(np.float32)
    temps = np.concatenate([rng.uniform(0.05, 2.0, 3000), rng.uniform(2, 30, 1500),
                            [1.0, 0.7, 1e-3, 1e3] * 250]).astype(np.float32)
    checked = 0
    for v, T in zip(vals, temps[:len(vals)]):
        if v == 0 or not np.isfinite(F32(v / T)) or abs(F32(v / T)) < 2.0 ** -120:
            continue
        assert fast_bound(v) <= exact_bound(v, T), (v, T)
        checked += 1
    assert checked > 4000
