"""Generate golden vectors from the reference sampler (apollo722/nano-inference).

Run in a container where the reference source is available::

    python tests/golden/make_golden.py --reference /path/to/nano-inference/src

It imports the unmodified ``nano_inference.sampling.sampler.Sampler`` and
records its outputs on seeded inputs (inputs are regenerated from the seeds by
the tests, with a checksum stored to detect generator drift):

* ``unit``      -- the reference's own known-answer tests
                   (``tests/unit/test_sampler.py:12-54``);
* ``penalty``   -- ``Sampler._apply_repetition_penalty`` (``sampler.py:93-108``)
                   values at every history id, as fp32 bit patterns;
* ``greedy``    -- ``Sampler.select_batch`` ids with temperature 0 (fp32 and
                   bf16 logits widened with ``.float()``);
* ``filter``    -- ``Sampler._apply_top_k_top_p`` (``sampler.py:110-133``)
                   survivor ids on ``x / T``;
* ``sampled``   -- ``Sampler.select_batch`` ids with ``torch.multinomial``
                   replaced by an inverse-CDF draw over the reference's own
                   probabilities (ascending token id, float64 running sum) from
                   fixed uniforms: the reference's draw is random, this pins
                   everything up to it.

The output (``reference_sampler.json``) is committed; the reference itself is
not needed to run the tests.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "nano-inference_b200"))

from b200_sampler.workloads import make_histories, make_logits, make_uniforms  # noqa: E402


def _checksum(t: torch.Tensor) -> float:
    return float(t.double().sum().item())


def _bits(v: float) -> int:
    return int(np.float32(v).view(np.uint32))


class InverseCdfDraw:
    """Stand-in for ``torch.multinomial(probs, 1)``: row r draws the first id
    whose float64 running sum of probs exceeds ``u[r] * total``."""

    def __init__(self, uniforms):
        self.u = [float(v) for v in uniforms]

    def __call__(self, probs, num_samples=1, *args, **kwargs):
        assert num_samples == 1
        P = probs.detach().double().numpy()
        out = []
        assert P.shape[0] == len(self.u), (P.shape, len(self.u))
        for r in range(P.shape[0]):
            c = np.cumsum(P[r])
            i = int(np.searchsorted(c, np.float32(self.u[r]) * c[-1], side="right"))
            out.append(min(i, P.shape[1] - 1))
        return torch.tensor(out, dtype=torch.long).unsqueeze(-1)


def gen(ref_src: str) -> dict:
    sys.path.insert(0, ref_src)
    from nano_inference.core.sampling import SamplingParams as RefParams
    from nano_inference.sampling.sampler import Sampler

    S = Sampler()
    out = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__}

    # ---- the reference's own known-answer tests -------------------------
    unit = []
    unit.append({"name": "greedy", "logits": [-1.0, 5.0, 2.0, -0.5], "history": [],
                 "temperature": 0.0, "rep": 1.0,
                 "token": S.select(torch.tensor([-1.0, 5.0, 2.0, -0.5]), [], RefParams(temperature=0.0))})
    unit.append({"name": "rep_off", "logits": [0.0, 10.0, 0.0], "history": [1],
                 "temperature": 0.0, "rep": 1.0,
                 "token": S.select(torch.tensor([0.0, 10.0, 0.0]), [1],
                                   RefParams(temperature=0.0, repetition_penalty=1.0))})
    unit.append({"name": "rep_100", "logits": [1.0, 10.0, 1.0], "history": [1],
                 "temperature": 0.0, "rep": 100.0,
                 "token": S.select(torch.tensor([1.0, 10.0, 1.0]), [1],
                                   RefParams(temperature=0.0, repetition_penalty=100.0))})
    keep = S._apply_top_k_top_p(torch.tensor([1.0, 2.0, 3.0, 4.0, 5.0]) / 1.0, top_k=2, top_p=1.0)
    unit.append({"name": "top_k2", "logits": [1.0, 2.0, 3.0, 4.0, 5.0], "temperature": 1.0,
                 "top_k": 2, "survivors": [int(i) for i in torch.nonzero(keep > -float("inf")).flatten()]})
    out["unit"] = unit

    # ---- repetition penalty, bit patterns --------------------------------
    pen = []
    V = 5003
    for seed, H, rep, dist in [(0, 64, 1.1, "uniform"), (1, 700, 1.2, "zipf"),
                               (2, 300, 0.8, "uniform"), (3, 50, 100.0, "uniform"),
                               (4, 200, 1.0, "uniform"), (5, 0, 1.3, "uniform"),
                               (6, 1, 1.3333333, "uniform")]:
        x = make_logits(seed, 1, V, 3.0)[0]
        h = make_histories(seed, 1, V, H, dist=dist)[0]
        y = S._apply_repetition_penalty(x.clone(), h, rep)
        uniq = sorted(set(h))
        pen.append({"seed": seed, "vocab": V, "scale": 3.0, "hist_len": H, "dist": dist, "rep": rep,
                    "checksum": _checksum(x), "ids": uniq,
                    "bits": [_bits(float(y[i])) for i in uniq],
                    "row_checksum": _checksum(y)})
    # exact zeros and signed zeros around the divide/multiply branch
    x = torch.tensor([0.0, -0.0, -1e-30, 1e-30, -3.0, 3.0, float("-inf"), float("inf")])
    h = list(range(8))
    y = S._apply_repetition_penalty(x.clone(), h, 1.7)
    pen.append({"explicit": [float(v) for v in x.tolist()], "rep": 1.7, "ids": h,
                "bits": [_bits(float(y[i])) for i in h]})
    out["penalty"] = pen

    # ---- greedy select_batch --------------------------------------------
    gr = []
    for seed, B, V, scale, rep, H, dt in [(10, 8, 5003, 3.0, 1.2, 128, "f32"),
                                         (11, 8, 4096, 2.0, 1.2, 512, "bf16"),
                                         (12, 4, 151936, 2.0, 1.2, 512, "bf16"),
                                         (13, 6, 333, 3.0, 1.0, 0, "f32")]:
        xt = make_logits(seed, B, V, scale, dtype=torch.bfloat16 if dt == "bf16" else torch.float32)
        hs = make_histories(seed, B, V, H, dist="zipf" if H > 100 else "uniform")
        params = [RefParams(temperature=0.0, repetition_penalty=rep) for _ in range(B)]
        ids = S.select_batch(xt.float().clone(), hs, params)
        gr.append({"seed": seed, "batch": B, "vocab": V, "scale": scale, "dtype": dt, "rep": rep,
                   "hist_len": H, "dist": "zipf" if H > 100 else "uniform",
                   "checksum": _checksum(xt.float()), "tokens": ids})
    out["greedy"] = gr

    # ---- top-k / top-p survivor sets ------------------------------------
    flt = []
    V = 5003
    x = make_logits(20, 1, V, 3.0)[0]
    for T in (0.7, 1.3):
        y = x / torch.tensor([T], dtype=torch.float32)
        for k in (-1, 0, 1, 2, 50, 200, V - 1, V, V + 5):
            for p in (1.0, 0.9, 0.5, 0.0, 0.97):
                if k in (-1, 0, V, V + 5) and p in (1.0, 0.0):
                    continue  # no filtering at all
                f = S._apply_top_k_top_p(y.clone(), top_k=k, top_p=p)
                surv = torch.nonzero(f > -float("inf")).flatten().tolist()
                flt.append({"seed": 20, "vocab": V, "scale": 3.0, "temperature": T, "top_k": k,
                            "top_p": p, "checksum": _checksum(x), "survivors": surv})
    # full-vocab headline rows
    xs = make_logits(21, 2, 151936, 3.0)
    for r in range(2):
        y = xs[r] / torch.tensor([0.7], dtype=torch.float32)
        f = S._apply_top_k_top_p(y.clone(), top_k=50, top_p=0.9)
        flt.append({"seed": 21, "row": r, "batch": 2, "vocab": 151936, "scale": 3.0, "temperature": 0.7,
                    "top_k": 50, "top_p": 0.9, "checksum": _checksum(xs),
                    "survivors": torch.nonzero(f > -float("inf")).flatten().tolist()})
    out["filter"] = flt

    # ---- sampled select_batch with an inverse-CDF draw ------------------
    smp = []
    real_multinomial = torch.multinomial
    try:
        for seed, B, V, spike, H, mixed in [(30, 16, 5003, 0.0, 64, False),
                                            (31, 16, 5003, 0.05, 256, True),
                                            (32, 4, 151936, 0.0, 1024, False)]:
            xt = make_logits(seed, B, V, 3.0, spike_frac=spike)
            hs = make_histories(seed, B, V, H)
            rng = np.random.default_rng(seed)
            plist = []
            for b in range(B):
                if seed == 32:
                    plist.append(dict(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1))
                else:
                    T = 0.0 if (mixed and b % 5 == 0) else float(rng.uniform(0.3, 1.5))
                    plist.append(dict(temperature=T, top_k=int(rng.choice([-1, 1, 5, 40, 200])),
                                      top_p=float(rng.choice([1.0, 0.95, 0.8, 0.5])),
                                      repetition_penalty=float(rng.choice([1.0, 1.1, 1.3]))))
            u = make_uniforms(seed + 100, B)
            sampled_rows = [b for b in range(B) if np.float32(plist[b]["temperature"]) != 0]
            torch.multinomial = InverseCdfDraw([u[b] for b in sampled_rows])
            ids = S.select_batch(xt.clone(), hs, [RefParams(**d) for d in plist])
            smp.append({"seed": seed, "batch": B, "vocab": V, "scale": 3.0, "spike_frac": spike,
                        "hist_len": H, "uniform_seed": seed + 100, "params": plist,
                        "checksum": _checksum(xt), "tokens": ids})
    finally:
        torch.multinomial = real_multinomial
    out["sampled"] = smp
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the reference's src/ directory")
    ap.add_argument("--out", default=os.path.join(HERE, "reference_sampler.json"))
    a = ap.parse_args()
    d = gen(a.reference)
    with open(a.out, "w") as f:
        json.dump(d, f, separators=(",", ":"))
    print("wrote", a.out, os.path.getsize(a.out), "bytes")


if __name__ == "__main__":
    main()
