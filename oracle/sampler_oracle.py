"""CPU oracle for the token-sampling path.  TEST INFRASTRUCTURE ONLY.

This module is the checker the CUDA sampler is compared against.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it; the product path (``b200_sampler``) never does, and fails loudly when
its CUDA library is missing.

It restates, in numpy, the reference sampler of apollo722/nano-inference
(``src/nano_inference/sampling/sampler.py``) plus three extensions that the
reference does not have and whose definitions live here:

* presence / frequency penalties (applied after the repetition penalty, each
  as a separately rounded fp32 operation);
* inverse-CDF sampling from a caller-supplied uniform ``u`` in place of
  ``torch.multinomial`` (``sampler.py:87``), whose RNG stream cannot be matched;
* the Philox4x32-10 uniform stream used when the caller passes no uniforms.

Arithmetic that the reference performs in fp32 is performed here in fp32 with
the same operation order, so penalised logits, ``logits / T`` and greedy
argmax are bit-exact (pinned against the reference by ``tests/golden``).
Softmax / cumsum / inverse-CDF sums are computed in float64; the GPU computes
them in a different order, so decisions that fall within ``EXEMPT_EPS`` of a
threshold are reported as *exempt* together with the set of acceptable ids.

Tie rule: the reference sorts with ``torch.sort`` (unstable on CPU, tie order
unspecified).  This oracle and the CUDA path both order equal logits by
ascending token id, so they agree on ties; only against the reference itself is
a tie group that straddles the top-p cut exempt (``RowResult.tie_at_cut``).

Philox4x32-10 is pinned by the Random123 known-answer vectors
(``tests/test_oracle.py``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

EXEMPT_EPS = 1e-6

_M0 = 0xD2511F53
_M1 = 0xCD9E8D57
_W0 = 0x9E3779B9
_W1 = 0xBB67AE85
_MASK32 = 0xFFFFFFFF


# --------------------------------------------------------------------------
# Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy
# as 1, 2, 3", SC'11).  Used for the default uniform stream; the CUDA kernel
# implements the same function.
# --------------------------------------------------------------------------
def philox4x32_10(ctr: Sequence[int], key: Sequence[int]) -> List[int]:
    c0, c1, c2, c3 = (int(v) & _MASK32 for v in ctr)
    k0, k1 = (int(v) & _MASK32 for v in key)
    for r in range(10):
        p0 = _M0 * c0
        p1 = _M1 * c2
        hi0, lo0 = (p0 >> 32) & _MASK32, p0 & _MASK32
        hi1, lo1 = (p1 >> 32) & _MASK32, p1 & _MASK32
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        if r < 9:
            k0 = (k0 + _W0) & _MASK32
            k1 = (k1 + _W1) & _MASK32
    return [c0, c1, c2, c3]


def philox_uniform(seed: int, offset: int, row: int) -> np.float32:
    """Uniform in [0, 1) for one batch row: counter = (row, offset), key = seed;
    the top 24 bits of the first output word, scaled by 2^-24."""
    ctr = (row & _MASK32, (row >> 32) & _MASK32, offset & _MASK32, (offset >> 32) & _MASK32)
    key = (seed & _MASK32, (seed >> 32) & _MASK32)
    w0 = philox4x32_10(ctr, key)[0]
    return np.float32((w0 >> 8) * (1.0 / 16777216.0))


def philox_uniforms(seed: int, offset: int, batch: int) -> np.ndarray:
    return np.array([philox_uniform(seed, offset, r) for r in range(batch)], dtype=np.float32)


# --------------------------------------------------------------------------
# dtype helpers
# --------------------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> exact fp32 values (the engine's ``.float()``,
    ``inferencer/torch_inferencer.py:249``)."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


def _get(p, name, default):
    return getattr(p, name, default) if p is not None else default


# --------------------------------------------------------------------------
# Penalties  (reference: sampler.py:93-108; presence/frequency: extension)
# --------------------------------------------------------------------------
def penalize_row(x: np.ndarray, hist: Sequence[int], rep: float,
                 pres: float = 0.0, freq: float = 0.0) -> np.ndarray:
    """Return penalised fp32 logits for one row.

    Repetition (sampler.py:99-107): skipped when ``rep == 1.0`` or the history
    is empty; for each *unique* history id, ``x * rep`` if ``x < 0`` else
    ``x / rep`` in fp32 (the Python float is rounded to fp32 first, as torch
    does for a 0-dim fp32 tensor op with a Python scalar).
    Extension: ``x = x - fp32(freq) * fp32(count)`` then ``x = x - fp32(pres)``,
    each rounded separately, with ``count`` the number of occurrences of the
    id in the same history.
    """
    x = np.array(x, dtype=np.float32, copy=True)
    if hist is None or len(hist) == 0:
        return x
    h = np.asarray(hist, dtype=np.int64)
    V = x.shape[0]
    if h.min() < 0 or h.max() >= V:
        raise IndexError("history token id out of range")
    ids, counts = np.unique(h, return_counts=True)
    if rep != 1.0:
        r = np.float32(rep)
        v = x[ids]
        x[ids] = np.where(v < 0, v * r, v / r).astype(np.float32)
    if freq != 0.0:
        x[ids] = (x[ids] - (np.float32(freq) * counts.astype(np.float32)).astype(np.float32)).astype(np.float32)
    if pres != 0.0:
        x[ids] = (x[ids] - np.float32(pres)).astype(np.float32)
    return x


def greedy_argmax(x: np.ndarray) -> int:
    """``torch.argmax`` semantics (sampler.py:70): first index of the maximum,
    NaN counts as the maximum (first NaN wins)."""
    return int(np.argmax(x))


# --------------------------------------------------------------------------
# Top-k / top-p  (reference: sampler.py:110-133)
# --------------------------------------------------------------------------
@dataclass
class TopPInfo:
    active: bool = False
    n_kept: int = 0
    exempt: bool = False
    order: Optional[np.ndarray] = None     # sorted positions (desc, ties by id)
    n_finite: int = 0
    tie_at_cut: bool = False


def top_k_keep(y: np.ndarray, k: int) -> np.ndarray:
    """Top-k mask (sampler.py:116-120): active iff ``0 < k < numel``; keeps
    every value ``>=`` the k-th largest (ties are all kept)."""
    V = y.shape[0]
    keep = np.ones(V, dtype=bool)
    if 0 < k < V:
        thr = np.partition(y, V - k)[V - k]
        keep = ~(y < thr)
    return keep


def _sorted_desc(f: np.ndarray) -> np.ndarray:
    # descending by value, ties by ascending index (stable)
    return np.argsort(-f, kind="stable")


def top_p_keep(y: np.ndarray, keep_k: np.ndarray, p: float, n_override: Optional[int] = None):
    """Top-p mask over the top-k survivors (sampler.py:122-131): sort
    descending, softmax, cumsum; remove sorted position ``j >= 1`` iff
    ``cumsum[j-1] > p``.  Active iff ``0 < fp32(p) < 1``.

    Returns (mask, TopPInfo).  ``n_override`` forces the number of kept sorted
    positions (used to enumerate the outcomes of an exempt decision).
    """
    p32 = np.float32(p)
    info = TopPInfo()
    if not (0.0 < p32 < 1.0):
        return keep_k.copy(), info
    info.active = True
    f = np.where(keep_k, y, np.float32(-np.inf)).astype(np.float32)
    finite = f > -np.inf
    n_fin = int(finite.sum())
    info.n_finite = n_fin
    # only finite entries carry mass; -inf entries sort last and change nothing
    cand = np.nonzero(finite)[0]
    sub = f[cand]
    o = _sorted_desc(sub)
    order = cand[o]
    info.order = order
    vals = f[order].astype(np.float64)
    if n_fin == 0:
        return np.zeros_like(keep_k), info
    e = np.exp(vals - vals[0])
    q = e / e.sum()
    cum = np.cumsum(q)
    pf = float(p32)
    if n_override is None:
        L = 1 + int(np.count_nonzero(cum[: n_fin - 1] <= pf))
    else:
        L = max(1, min(n_fin, n_override))
    info.n_kept = L
    near = np.abs(cum[: n_fin - 1] - pf) <= EXEMPT_EPS
    # torch.sort's tie order is unspecified: against the reference itself a tie
    # group straddling the cut may be kept differently (the CUDA path and this
    # oracle share the ascending-id rule, so it is not an exemption between them)
    info.tie_at_cut = bool(L < n_fin and vals[L - 1] == vals[L])
    info.exempt = bool(near.any())
    mask = np.zeros_like(keep_k)
    mask[order[:L]] = True
    return mask, info


def inverse_cdf(y: np.ndarray, keep: np.ndarray, u: float):
    """Draw one token from softmax(y) restricted to ``keep``: the first kept id,
    in ascending id order, whose running sum of ``exp(y - max)`` exceeds
    ``u * total`` (extension replacing torch.multinomial, sampler.py:86-89).

    Returns (token, exempt, neighbours)."""
    ids = np.nonzero(keep & (y > -np.inf))[0]
    if ids.size == 0:
        raise FloatingPointError("no finite survivor")
    yv = y[ids].astype(np.float64)
    w = np.exp(yv - yv.max())
    prefix = np.cumsum(w)
    total = prefix[-1]
    target = float(np.float32(u)) * total
    i = int(np.searchsorted(prefix, target, side="right"))
    if i >= ids.size:
        i = ids.size - 1
    tol = EXEMPT_EPS * total
    exempt = abs(prefix[i] - target) <= tol or (i > 0 and abs(prefix[i - 1] - target) <= tol)
    neigh = {int(ids[j]) for j in (i - 1, i, i + 1) if 0 <= j < ids.size}
    return int(ids[i]), bool(exempt), neigh


# --------------------------------------------------------------------------
# Whole-row and batch entry points
# --------------------------------------------------------------------------
@dataclass
class RowResult:
    token: int = -1
    error: bool = False          # reference raises (NaN / inf probabilities)
    exempt: bool = False         # a decision within EXEMPT_EPS of a threshold
    allowed: set = field(default_factory=set)   # acceptable ids when exempt
    greedy: bool = False
    n_topk: int = 0              # survivors after top-k
    n_kept: int = 0              # survivors after top-p
    tie_at_cut: bool = False     # equal logits straddle the top-p cut


def sample_row(x: np.ndarray, hist: Sequence[int], params, u: float) -> RowResult:
    """One row of ``Sampler.select_batch`` (sampler.py:36-91) with the
    inverse-CDF draw.  ``x`` is the fp32 row (bf16 already widened)."""
    rep = float(_get(params, "repetition_penalty", 1.0))
    pres = float(_get(params, "presence_penalty", 0.0) or 0.0)
    freq = float(_get(params, "frequency_penalty", 0.0) or 0.0)
    T = float(_get(params, "temperature", 0.7))
    k = int(_get(params, "top_k", -1))
    p = float(_get(params, "top_p", 1.0))
    res = RowResult()
    xp = penalize_row(x, hist, rep, pres, freq)
    T32 = np.float32(T)
    if T32 == 0:                       # sampler.py:60-70 (temperatures in logits dtype)
        res.greedy = True
        res.token = greedy_argmax(xp)
        res.allowed = {res.token}
        return res
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        y = (xp / T32).astype(np.float32)          # sampler.py:73-76
    if np.isnan(y).any() or np.isposinf(y).any() or not (y > -np.inf).any():
        res.error = True
        return res
    keep_k = top_k_keep(y, k)
    res.n_topk = int(np.count_nonzero(keep_k & (y > -np.inf)))
    keep, info = top_p_keep(y, keep_k, p)
    res.n_kept = int(np.count_nonzero(keep & (y > -np.inf)))
    tok, ex_cdf, neigh = inverse_cdf(y, keep, u)
    res.token = tok
    res.allowed = {tok} | (neigh if ex_cdf else set())
    res.exempt = ex_cdf
    res.tie_at_cut = bool(info.active and info.tie_at_cut)
    if info.active and info.exempt:
        res.exempt = True
        L = info.n_kept
        for L2 in (L - 1, L + 1):
            if 1 <= L2 <= info.n_finite:
                m2, _ = top_p_keep(y, keep_k, p, n_override=L2)
                t2, _, n2 = inverse_cdf(y, m2, u)
                res.allowed |= {t2} | n2
    return res


def sample_batch(logits: np.ndarray, histories: Sequence[Sequence[int]], params: Sequence,
                 uniforms: Optional[np.ndarray] = None, seed: int = 0, offset: int = 0):
    """Batch oracle.  ``logits`` fp32 [B, V]; returns a list of RowResult."""
    B = logits.shape[0]
    if uniforms is None:
        uniforms = philox_uniforms(seed, offset, B)
    out = []
    for b in range(B):
        h = histories[b] if histories is not None else []
        out.append(sample_row(np.asarray(logits[b], dtype=np.float32), h, params[b], float(uniforms[b])))
    return out


def tokens(results: Sequence[RowResult]) -> List[int]:
    return [r.token for r in results]
