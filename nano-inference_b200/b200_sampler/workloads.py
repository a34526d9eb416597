"""Seeded synthetic inputs for the sampling path.

The reference publishes no benchmark data; these generators make the shapes,
value distributions and seeds of the benchmark configurations concrete.
Logits are drawn on the CPU with ``torch.Generator().manual_seed(seed)`` so
that the CUDA path and the CPU oracle see identical bytes; histories use
``numpy.random.default_rng(seed)``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

from .params import SamplingParams

QWEN_VOCAB = 151936


def make_logits(seed: int, batch: int, vocab: int, scale: float = 3.0,
                spike_frac: float = 0.0, spike: float = 15.0,
                dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """``randn * scale`` (optionally ``+spike`` on a ``rand < spike_frac`` mask),
    generated in fp32 on the CPU and then cast to ``dtype``."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, vocab, generator=g, dtype=torch.float32) * scale
    if spike_frac > 0:
        m = torch.rand(batch, vocab, generator=g) < spike_frac
        x = x + m.to(torch.float32) * spike
    return x.to(dtype)


def make_histories(seed: int, batch: int, vocab: int, length: int,
                   dist: str = "uniform", zipf_s: float = 1.1) -> List[List[int]]:
    """Per-row token histories (prompt + outputs): uniform ids in ``[0, vocab)``
    or a truncated Zipf law ``p(i) ~ (i + 1)^-s``."""
    rng = np.random.default_rng(seed)
    if length <= 0:
        return [[] for _ in range(batch)]
    if dist == "uniform":
        h = rng.integers(0, vocab, size=(batch, length))
    elif dist == "zipf":
        w = (np.arange(vocab, dtype=np.float64) + 1.0) ** (-zipf_s)
        w /= w.sum()
        h = rng.choice(vocab, size=(batch, length), p=w)
    else:
        raise ValueError(dist)
    return [list(map(int, r)) for r in h]


def make_uniforms(seed: int, batch: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.rand(batch, generator=g, dtype=torch.float32)


@dataclass
class Workload:
    name: str
    batch: int
    vocab: int
    logits: torch.Tensor                 # CPU, fp32 or bf16
    histories: List[List[int]]
    params: List[SamplingParams]
    uniforms: torch.Tensor               # CPU fp32 [batch]
    notes: str = ""
    meta: dict = field(default_factory=dict)

    @property
    def history_len(self) -> int:
        return max((len(h) for h in self.histories), default=0)


def headline(batch: int = 256, vocab: int = QWEN_VOCAB, seed: int = 0) -> Workload:
    """North-star headline: B=256, V=151936 fp32 ``randn*3``; T=0.7, top-k 50,
    top-p 0.9, repetition 1.1, presence 0.5, frequency 0.3; 1024 uniform
    history ids per row; uniforms from seed 1."""
    p = SamplingParams(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1,
                       presence_penalty=0.5, frequency_penalty=0.3)
    return Workload("headline", batch, vocab, make_logits(seed, batch, vocab, 3.0),
                    make_histories(seed, batch, vocab, 1024), [p] * batch,
                    make_uniforms(1, batch),
                    notes="B=%d V=%d fp32 randn*3 T=0.7 k=50 p=0.9 rep=1.1 pres=0.5 freq=0.3 H=1024"
                    % (batch, vocab))


def config1(seed: int = 0) -> Workload:
    """C1: B=8 fp32 ``randn*3``; T=0.7, k=50, p=0.9, rep 1.1; 64 uniform ids."""
    B, V = 8, QWEN_VOCAB
    p = SamplingParams(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1)
    return Workload("c1", B, V, make_logits(seed, B, V, 3.0), make_histories(seed, B, V, 64),
                    [p] * B, make_uniforms(1, B))


def config2(seed: int = 0, batch: int = 64) -> Workload:
    """C2: greedy + penalties, bf16 ``randn*2``; presence 0.5, frequency 0.3,
    repetition 1.2 over 512 Zipf(1.1) ids."""
    V = QWEN_VOCAB
    p = SamplingParams(temperature=0.0, repetition_penalty=1.2, presence_penalty=0.5,
                       frequency_penalty=0.3)
    return Workload("c2", batch, V, make_logits(seed, batch, V, 2.0, dtype=torch.bfloat16),
                    make_histories(seed, batch, V, 512, dist="zipf"), [p] * batch,
                    make_uniforms(1, batch))


def config3(seed: int = 0, batch: int = 256) -> Workload:
    """C3: heterogeneous batch; fp32 ``randn*3`` + 5% spikes of +15; per-row
    T~U[0.3,1.5], k~U{1..200}, p~U[0.5,1.0]; rep 1.1, pres 0.5, freq 0.3;
    1024 uniform ids."""
    V = QWEN_VOCAB
    rng = np.random.default_rng(seed + 7)
    params = [SamplingParams(temperature=float(rng.uniform(0.3, 1.5)),
                             top_k=int(rng.integers(1, 201)),
                             top_p=float(rng.uniform(0.5, 1.0)),
                             repetition_penalty=1.1, presence_penalty=0.5,
                             frequency_penalty=0.3) for _ in range(batch)]
    return Workload("c3", batch, V, make_logits(seed, batch, V, 3.0, spike_frac=0.05),
                    make_histories(seed, batch, V, 1024), params, make_uniforms(1, batch))


def config4(seed: int = 0, batch: int = 128) -> Workload:
    """C4 (vocab-parallel): fp32 ``randn*3``; k=50, p=0.95, T=0.8; no penalties."""
    V = QWEN_VOCAB
    p = SamplingParams(temperature=0.8, top_k=50, top_p=0.95)
    return Workload("c4", batch, V, make_logits(seed, batch, V, 3.0),
                    [[] for _ in range(batch)], [p] * batch, make_uniforms(1, batch))


def topp095(seed: int = 0, batch: int = 256) -> Workload:
    """Top-p only (top-k off), p 0.95, T 1.0, no penalties: the common
    production setting, fp32 ``randn*3``."""
    V = QWEN_VOCAB
    p = SamplingParams(temperature=1.0, top_p=0.95)
    return Workload("topp095", batch, V, make_logits(seed, batch, V, 3.0), [[] for _ in range(batch)],
                    [p] * batch, make_uniforms(1, batch),
                    notes="B=%d V=%d fp32 randn*3 T=1.0 top-k off p=0.95, no penalties" % (batch, V))


def softmax_only(seed: int = 0, batch: int = 256) -> Workload:
    """Plain multinomial draw: T 1.0, top-k and top-p off, no penalties."""
    V = QWEN_VOCAB
    p = SamplingParams(temperature=1.0)
    return Workload("softmax", batch, V, make_logits(seed, batch, V, 3.0), [[] for _ in range(batch)],
                    [p] * batch, make_uniforms(1, batch),
                    notes="B=%d V=%d fp32 randn*3 T=1.0, top-k / top-p off, no penalties" % (batch, V))


def k240(seed: int = 0, batch: int = 256) -> Workload:
    """The headline with top-k 240 (the largest single-pass top-k)."""
    w = headline(batch=batch, seed=seed)
    p = SamplingParams(temperature=0.7, top_k=240, top_p=0.9, repetition_penalty=1.1,
                       presence_penalty=0.5, frequency_penalty=0.3)
    w.name, w.params = "k240", [p] * batch
    w.notes = w.notes.replace("k=50", "k=240")
    return w


def _with_notes(w: Workload, notes: str) -> Workload:
    w.notes = notes
    return w


# Named workloads of the benchmark (``bench.py --workload``).
WORKLOADS = {
    "headline": lambda: headline(),
    "c1": lambda: _with_notes(config1(), "C1: B=8 V=151936 fp32 randn*3 T=0.7 k=50 p=0.9 rep=1.1 H=64"),
    "c2": lambda: _with_notes(config2(), "C2: B=64 V=151936 bf16 randn*2 greedy, rep=1.2 pres=0.5 freq=0.3, "
                                         "H=512 Zipf(1.1)"),
    "c3": lambda: _with_notes(config3(), "C3: B=256 V=151936 fp32 randn*3 + 5% spikes, per-row T U[0.3,1.5] "
                                         "k U{1..200} p U[0.5,1], rep=1.1 pres=0.5 freq=0.3, H=1024"),
    "topp095": lambda: topp095(),
    "softmax": lambda: softmax_only(),
    "k240": lambda: k240(),
}
