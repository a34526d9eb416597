"""Parity at the exact shapes the benchmark and the benchmark configurations
run, through the C ABI, against the CPU oracle.

The launch shape depends on the batch: from 148 rows up (the SM count) every
row runs on one block, below that rows are split over 2-8 block clusters.  The
headline (B=256, one block per row, top-k 50 with 1024-id penalties) and
config 3 (B=256, heterogeneous top-k / top-p / T) are therefore checked at their
full batch, config 1 at its B=8 (8-block clusters) and config 2 at B=64.

Acceptance as in test_gpu_sampler: greedy rows bit-exact; sampled rows equal
unless the oracle marks the row exempt (a top-p cumsum or an inverse-CDF step
within 1e-6 of its threshold), in which case the id must be one of the
oracle's alternatives.
"""
import numpy as np
import pytest
import torch

from oracle import sampler_oracle as O
from b200_sampler.params import SamplingParams
from b200_sampler.workloads import config1, config2, config3, headline, make_histories, make_logits, make_uniforms

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sampler():
    from b200_sampler import B200Sampler
    return B200Sampler(seed=4321)


def _check(ids, ref, ctx):
    n_exempt = 0
    for b, r in enumerate(ref):
        if r.error:
            assert ids[b] < 0, (ctx, b, ids[b])
            continue
        if ids[b] != r.token:
            assert r.exempt and ids[b] in r.allowed, (ctx, b, ids[b], r.token, r.exempt)
            n_exempt += 1
    return n_exempt


def _run(sampler, w):
    ids = sampler.select_batch_tensor(w.logits.cuda(), w.histories, w.params,
                                      uniforms=w.uniforms.cuda()).cpu().tolist()
    ref = O.sample_batch(w.logits.float().numpy(), w.histories, w.params, uniforms=w.uniforms.numpy())
    return ids, ref


@pytest.mark.parametrize("seed", [0, 1])
def test_headline_full_batch_one_block_per_row(sampler, seed):
    """The benchmarked launch: 256 rows x 151936 fp32, T 0.7, k 50, p 0.9,
    repetition 1.1, presence 0.5, frequency 0.3 over 1024 uniform ids."""
    w = headline(batch=256, seed=seed)
    ids, ref = _run(sampler, w)
    assert _check(ids, ref, f"headline seed {seed}") <= 3


def test_config3_full_batch(sampler):
    w = config3(batch=256)
    ids, ref = _run(sampler, w)
    assert _check(ids, ref, "config3 B=256") <= 3


def test_config1_batch8_clusters(sampler):
    w = config1()
    ids, ref = _run(sampler, w)
    assert _check(ids, ref, "config1") <= 1


def test_config2_greedy_bit_exact(sampler):
    w = config2(batch=64)
    ids, ref = _run(sampler, w)
    assert ids == [r.token for r in ref]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_top_k_225_to_240_one_block_per_row(sampler, dtype):
    """One block per row (160 rows) with top-k 225..240: the windowed top-k
    path.  Rows with penalties and negative temperatures, and rows whose tie
    run at the k-th value is the smallest value collected by the window (a
    plateau of 40 equal values straddling rank k with a deep gap below it), so
    the run reaches the last collected key."""
    B, V = 160, 151936
    x = make_logits(211, B, V, 3.0)
    order = torch.argsort(x, dim=1, descending=True)
    plateau_rows = list(range(0, B, 8))
    for b in plateau_rows:
        idx = order[b]
        x[b, idx[210:250]] = float(x[b, idx[210]])
        x[b, idx[250:]] -= 6.0 if b % 16 == 0 else 1.5
    x = x.to(dtype)
    hs = make_histories(212, B, V, 512)
    rng = np.random.default_rng(213)
    params = []
    for b in range(B):
        pen = dict(repetition_penalty=1.1, presence_penalty=0.5, frequency_penalty=0.3) if b % 2 else {}
        t = float(rng.choice([0.7, 1.0, -0.8, 1.3]))
        k = int(rng.choice([225, 228, 232, 236, 240]))
        p = float(rng.choice([1.0, 0.9, 0.95]))
        if b in plateau_rows:
            t, k = 1.0, 230
        params.append(SamplingParams(temperature=t, top_k=k, top_p=p, **pen))
    u = make_uniforms(214, B)
    ids = sampler.select_batch_tensor(x.cuda(), hs, params, uniforms=u.cuda()).cpu().tolist()
    ref = O.sample_batch(x.float().numpy(), hs, params, uniforms=u.numpy())
    assert _check(ids, ref, f"k 225..240 {dtype}") <= 4


def test_last_position_of_a_bsv_tensor_in_place(sampler):
    """The decode step's feed: ``logits[:, -1, :]`` of a bf16 [B, S, V] model
    output, read in place through the row stride S x V (the reference stacks
    ``.float()`` copies of these rows, inferencer/torch_inferencer.py:242-251)."""
    B, S, V = 16, 5, 151936
    full = make_logits(400, B * S, V, 2.0).view(B, S, V).to(torch.bfloat16).cuda()
    x = full[:, -1, :]
    assert x.stride() == (S * V, 1)
    hs = make_histories(401, B, V, 300)
    params = [SamplingParams(temperature=0.7, top_k=20, top_p=0.8, repetition_penalty=1.1) if b % 3
              else SamplingParams(temperature=0.0, repetition_penalty=1.2) for b in range(B)]
    u = make_uniforms(402, B)
    ids = sampler.select_batch_tensor(x, hs, params, uniforms=u.cuda()).cpu().tolist()
    ref = O.sample_batch(x.float().cpu().numpy(), hs, params, uniforms=u.numpy())
    assert _check(ids, ref, "[B,S,V] last position") <= 1
