"""Load ``reference_sampler.json`` and regenerate the inputs of each case."""
from __future__ import annotations

import json
import os
from functools import lru_cache

import numpy as np
import torch

from b200_sampler.params import SamplingParams
from b200_sampler.workloads import make_histories, make_logits, make_uniforms

HERE = os.path.dirname(os.path.abspath(__file__))


@lru_cache(maxsize=1)
def golden() -> dict:
    with open(os.path.join(HERE, "reference_sampler.json")) as f:
        return json.load(f)


def _check(t: torch.Tensor, checksum: float):
    got = float(t.double().sum().item())
    assert got == checksum, f"input generator drift: checksum {got} != {checksum}"


def penalty_inputs(case):
    x = make_logits(case["seed"], 1, case["vocab"], case["scale"])
    _check(x[0], case["checksum"])
    h = make_histories(case["seed"], 1, case["vocab"], case["hist_len"], dist=case["dist"])[0]
    return x[0].numpy(), h


def greedy_inputs(case):
    dt = torch.bfloat16 if case["dtype"] == "bf16" else torch.float32
    x = make_logits(case["seed"], case["batch"], case["vocab"], case["scale"], dtype=dt)
    _check(x.float(), case["checksum"])
    hs = make_histories(case["seed"], case["batch"], case["vocab"], case["hist_len"], dist=case["dist"])
    params = [SamplingParams(temperature=0.0, repetition_penalty=case["rep"])] * case["batch"]
    return x, hs, params


def filter_inputs(case):
    if "row" in case:
        x = make_logits(case["seed"], case["batch"], case["vocab"], case["scale"])
        _check(x, case["checksum"])
        return x[case["row"]].numpy()
    x = make_logits(case["seed"], 1, case["vocab"], case["scale"])
    _check(x[0], case["checksum"])
    return x[0].numpy()


def sampled_inputs(case):
    x = make_logits(case["seed"], case["batch"], case["vocab"], case["scale"], spike_frac=case["spike_frac"])
    _check(x, case["checksum"])
    hs = make_histories(case["seed"], case["batch"], case["vocab"], case["hist_len"])
    params = [SamplingParams(**d) for d in case["params"]]
    u = make_uniforms(case["uniform_seed"], case["batch"])
    return x, hs, params, u


def f32_from_bits(bits):
    return np.array(bits, dtype=np.uint32).view(np.float32)
