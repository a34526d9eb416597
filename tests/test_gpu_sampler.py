"""Parity of the CUDA sampler with the CPU oracle (and the reference's golden
vectors), through the drop-in ``B200Sampler`` API and the C ABI.

Acceptance (per row): greedy and penalty-only rows bit-exact; sampled rows
identical unless the oracle marks the row exempt (a top-p cumsum or an
inverse-CDF step within EXEMPT_EPS = 1e-6 of its threshold), in which case the
id must be one of the oracle's alternatives.
"""
import numpy as np
import pytest
import torch

from oracle import sampler_oracle as O
from b200_sampler.params import SamplingParams
from b200_sampler.workloads import make_histories, make_logits, make_uniforms
from golden.fixtures import golden, greedy_inputs, sampled_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sampler():
    from b200_sampler import B200Sampler
    return B200Sampler(seed=1234)


def check(got, ref, ctx=""):
    n_exempt = 0
    for b, r in enumerate(ref):
        if r.error:
            assert got[b] < 0, (ctx, b, got[b])
            continue
        if got[b] != r.token:
            assert r.exempt and got[b] in r.allowed, (ctx, b, got[b], r.token, r.exempt)
            n_exempt += 1
    return n_exempt


def run(sampler, x, hs, params, u, dev_logits=None):
    """GPU ids (negative entries = failed rows) and oracle results."""
    xl = dev_logits if dev_logits is not None else x.cuda()
    ids = sampler.select_batch_tensor(xl, hs, params, uniforms=u.cuda()).cpu().tolist()
    ref = O.sample_batch(x.float().numpy(), hs, params, uniforms=u.numpy())
    return ids, ref


# --------------------------------------------------------------------------
# the reference's own unit tests (tests/unit/test_sampler.py)
# --------------------------------------------------------------------------
def test_reference_unit_greedy(sampler):
    p = SamplingParams(temperature=0.0)
    assert sampler.select(torch.tensor([-1.0, 5.0, 2.0, -0.5]), [], p) == 1


def test_reference_unit_repetition_penalty(sampler):
    p = SamplingParams(temperature=0.0, repetition_penalty=1.0)
    assert sampler.select(torch.tensor([0.0, 10.0, 0.0]), [1], p) == 1
    p = SamplingParams(temperature=0.0, repetition_penalty=100.0)
    assert sampler.select(torch.tensor([1.0, 10.0, 1.0]), [1], p) in (0, 2)


def test_reference_unit_top_k(sampler):
    p = SamplingParams(temperature=1.0, top_k=2)
    x = torch.tensor([1.0, 2.0, 3.0, 4.0, 5.0])
    sel = {sampler.select(x, [], p) for _ in range(20)}
    assert sel.issubset({3, 4})
    u = torch.linspace(0, 0.999, 64)
    sel = {sampler.select(x, [], p, uniforms=u[i:i + 1]) for i in range(64)}
    assert sel == {3, 4}


# --------------------------------------------------------------------------
# golden vectors produced by the reference sampler
# --------------------------------------------------------------------------
def test_golden_greedy(sampler):
    for case in golden()["greedy"]:
        x, hs, params = greedy_inputs(case)
        got = sampler.select_batch(x.cuda(), hs, params)
        assert got == case["tokens"], case["seed"]


def test_golden_sampled(sampler):
    for case in golden()["sampled"]:
        x, hs, params, u = sampled_inputs(case)
        got = sampler.select_batch(x.cuda(), hs, params, uniforms=u.cuda())
        ref = O.sample_batch(x.numpy(), hs, params, uniforms=u.numpy())
        for b in range(case["batch"]):
            if got[b] != case["tokens"][b]:
                assert ref[b].exempt or ref[b].tie_at_cut, (case["seed"], b)


# --------------------------------------------------------------------------
# parity with the oracle
# --------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,V", [(1, 3), (3, 5), (4, 100), (5, 4099), (8, 32000), (16, 151936)])
def test_parity_mixed_rows(sampler, dtype, B, V):
    seed = B * 1000 + V
    x = make_logits(seed, B, V, 3.0, spike_frac=0.02, dtype=dtype)
    hs = make_histories(seed, B, V, min(V, 300))
    rng = np.random.default_rng(seed)
    params = []
    for b in range(B):
        kind = b % 4
        if kind == 0:
            params.append(SamplingParams(temperature=0.0, repetition_penalty=1.2, presence_penalty=0.5,
                                         frequency_penalty=0.3))
        else:
            params.append(SamplingParams(temperature=float(rng.uniform(0.3, 1.5)),
                                         top_k=int(rng.choice([1, 2, 20, 50, 200, 512])),
                                         top_p=float(rng.choice([1.0, 0.9, 0.5, 0.0])),
                                         repetition_penalty=float(rng.choice([1.0, 1.1, 0.9])),
                                         presence_penalty=float(rng.choice([0.0, 0.5])),
                                         frequency_penalty=float(rng.choice([0.0, 0.3, -0.2]))))
    u = make_uniforms(seed + 1, B)
    ids, ref = run(sampler, x, hs, params, u)
    check(ids, ref, f"{dtype} {B}x{V}")


def test_parity_headline_full_size(sampler):
    from b200_sampler.workloads import headline
    w = headline(batch=64)
    ids, ref = run(sampler, w.logits, w.histories, w.params, w.uniforms)
    n_ex = check(ids, ref, "headline")
    assert n_ex <= 2


def test_parity_config3_heterogeneous(sampler):
    from b200_sampler.workloads import config3
    w = config3(batch=48)
    ids, ref = run(sampler, w.logits, w.histories, w.params, w.uniforms)
    assert check(ids, ref, "c3") <= 2


def test_parity_config2_greedy_bf16_bit_exact(sampler):
    from b200_sampler.workloads import config2
    w = config2(batch=64)
    ids, ref = run(sampler, w.logits, w.histories, w.params, w.uniforms)
    assert ids == [r.token for r in ref]


def test_layouts_strided_and_misaligned(sampler):
    B, V = 6, 7001
    big = make_logits(77, B, V + 9, 3.0)
    hs = make_histories(77, B, V, 64)
    params = [SamplingParams(temperature=0.8, top_k=40, top_p=0.9, repetition_penalty=1.1)] * B
    u = make_uniforms(78, B)
    dev = big.cuda()
    for off in (0, 1, 2, 3):
        view = dev[:, off:off + V]                        # row stride V+9, base offset off
        x = big[:, off:off + V].contiguous()
        ids, ref = run(sampler, x, hs, params, u, dev_logits=view)
        check(ids, ref, f"offset {off}")


def test_negative_temperature_and_ties(sampler):
    B, V = 4, 5000
    x = torch.zeros(B, V)
    x[0, 100:110] = 1.0                      # tie group larger than k
    x[1] = torch.arange(V, dtype=torch.float32) % 7
    x[2] = make_logits(3, 1, V)[0]
    x[3] = make_logits(4, 1, V)[0]
    params = [SamplingParams(temperature=1.0, top_k=5),
              SamplingParams(temperature=0.7, top_k=3, top_p=0.5),
              SamplingParams(temperature=-0.7, top_k=10, top_p=0.9),
              SamplingParams(temperature=1e-3, top_k=50, top_p=0.95)]
    u = make_uniforms(9, B)
    ids, ref = run(sampler, x, [[]] * B, params, u)
    check(ids, ref, "ties")


@pytest.mark.parametrize("n_ties,K,B", [(300, 100, 2), (1500, 100, 2), (1500, 100, 200)])
def test_tie_plateau_merge_paths(sampler, n_ties, K, B):
    """A plateau of equal maxima larger than K: every tie is kept (reference
    top-k keeps values equal to the k-th).  300 ties reach the rank-sort merge
    with more than 128 kept survivors; 1500 exceed the rank-sort capacity, in
    cluster (B=2) and single-block (B=200) launches."""
    V = 151936
    rng = np.random.default_rng(n_ties * 7 + B)
    x = make_logits(n_ties + B, B, V, 1.0)
    for b in range(B):
        x[b, rng.choice(V, n_ties, replace=False)] = 9.0
    params = [SamplingParams(temperature=1.0, top_k=K, top_p=0.95)] * B
    u = make_uniforms(n_ties + 1, B)
    ids, ref = run(sampler, x, [[]] * B, params, u)
    check(ids, ref, f"ties {n_ties} B={B}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B", [8, 96, 160])
def test_softmax_rows_top_k_and_top_p_off(sampler, dtype, B):
    """The reference's default request (top_k -1, top_p 1.0): the draw is over
    the whole softmax, in one pass.  160 full-size rows (more than the SMs) run
    one block per row; 96 rows run 2-block clusters and 8 rows 8-block
    clusters, which exchange their maxima and masses.  k 0 or >= V and p 0.0
    also disable the filters."""
    V = 151936
    x = make_logits(61, B, V, 3.0, spike_frac=0.005, dtype=dtype)
    hs = make_histories(62, B, V, 256)
    rng = np.random.default_rng(63)
    params = []
    for b in range(B):
        pen = dict(repetition_penalty=1.2, presence_penalty=0.5, frequency_penalty=0.3) if b % 2 else {}
        params.append(SamplingParams(temperature=float(rng.choice([0.7, 1.3, -0.8, 0.05])),
                                     top_k=int(rng.choice([-1, 0, V, V + 5])),
                                     top_p=float(rng.choice([1.0, 0.0])), **pen))
    x[3, 1000] = float("nan")                  # an error row
    xf = x.float()
    xf[5, 77] = 3.0e38                         # x / T overflows for T < 1
    params[5] = SamplingParams(temperature=0.7, top_k=-1, top_p=1.0)
    u = make_uniforms(64, B)
    x_in = xf.to(dtype) if dtype == torch.float32 else x
    ids, ref = run(sampler, x_in, hs, params, u)
    assert check(ids, ref, f"softmax {dtype}") <= 3
    assert ids[3] < 0 and (dtype != torch.float32 or ids[5] < 0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cluster_union_past_1024_keys(sampler, dtype):
    """Eight rows run 8-block clusters; with k up to 240 each block keeps its
    own top-k with ties, so the leader's union of the eight lists exceeds 1024
    keys: the lists are staged whole and the first 1024 positions placed.  A
    row with a tie plateau larger than k checks the overflow rule."""
    B, V = 8, 151936
    x = make_logits(91, B, V, 3.0, dtype=torch.float32)
    x[5, 1000:1400] = x[5].max() + 1.0        # 400 equal leaders, k = 240: ties past the k-th
    x = x.to(dtype)
    hs = make_histories(92, B, V, 300)
    params = [SamplingParams(temperature=float(t), top_k=int(k), top_p=float(p),
                             repetition_penalty=1.1, presence_penalty=0.3)
              for t, k, p in [(0.7, 200, 0.9), (1.0, 240, 1.0), (0.5, 150, 0.95), (-0.8, 230, 0.8),
                              (1.3, 240, 0.99), (0.7, 240, 1.0), (0.9, 180, 0.5), (1.1, 129, 0.9)]]
    u = make_uniforms(93, B)
    ids, ref = run(sampler, x, hs, params, u)
    assert check(ids, ref, f"cluster union {dtype}") <= 2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B", [12, 96, 160])
def test_nucleus_rows_top_k_off(sampler, dtype, B):
    """Top-k off with top-p on.  The stream keeps the 128 largest as
    candidates and checks they hold more than p of the row's mass.  One block
    per row (160 rows): larger nuclei take one more pass (a plateau of 300
    near-equal leaders), and a nucleus past the key capacity (a flat row) the
    multi-pass path.  Clusters (96 rows: 2 blocks, 12 rows: 8 blocks) check the
    merged candidates against the mass rebuilt from every block, and take the
    multi-pass path when they fall short."""
    V = 151936
    x = make_logits(71, B, V, 3.0, spike_frac=0.005, dtype=torch.float32)
    x[7] = torch.randn(V, generator=torch.Generator().manual_seed(7)) * 0.01    # nucleus ~ 0.9 V
    x[9, :300] = 8.0 + torch.arange(300, dtype=torch.float32) * 1e-3            # ~300 near-equal leaders
    x = x.to(dtype)
    hs = make_histories(72, B, V, 256)
    rng = np.random.default_rng(73)
    params = []
    for b in range(B):
        pen = dict(repetition_penalty=1.1, presence_penalty=0.4, frequency_penalty=0.2) if b % 3 == 0 else {}
        params.append(SamplingParams(temperature=float(rng.choice([0.7, 1.0, -0.9, 1.5])),
                                     top_k=int(rng.choice([-1, 0, V])),
                                     top_p=float(rng.choice([0.5, 0.9, 0.95, 0.99])), **pen))
    params[7] = SamplingParams(temperature=1.0, top_k=-1, top_p=0.9)
    params[9] = SamplingParams(temperature=1.0, top_k=-1, top_p=0.9)
    u = make_uniforms(74, B)
    ids, ref = run(sampler, x, hs, params, u)
    assert check(ids, ref, f"nucleus {dtype}") <= 3


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_wide_top_k_rows(sampler, dtype):
    """Top-k between 241 and 2048 (one block per row): the stream keeps the 240
    largest, one more pass counts and collects a window below the row's
    maximum, and the finalise keeps the top-k with ties; a plateau of equal
    values at the k-th, a plateau above it, negative temperatures and
    penalised history columns in the window."""
    B, V = 160, 151936
    x = make_logits(101, B, V, 3.0, dtype=torch.float32)
    top = x.max(dim=1).values
    x[4, 7::211] = top[4] - 1.0                   # ~720 equal values near the top
    x[9, 3::97] = top[9] - 2.5                    # ~1566 equal values around the k-th
    x = x.to(dtype)
    hs = make_histories(102, B, V, 400)
    rng = np.random.default_rng(103)
    params = []
    for b in range(B):
        pen = dict(repetition_penalty=1.1, presence_penalty=0.3, frequency_penalty=0.1) if b % 2 else {}
        params.append(SamplingParams(temperature=float(rng.choice([0.5, 0.7, 1.0, -0.8, 1.3])),
                                     top_k=int(rng.choice([241, 300, 500, 1000, 1500, 2048])),
                                     top_p=float(rng.choice([1.0, 0.9, 0.5, 0.99])), **pen))
    params[4] = SamplingParams(temperature=1.0, top_k=300, top_p=1.0)
    params[9] = SamplingParams(temperature=1.0, top_k=1000, top_p=0.95)
    u = make_uniforms(104, B)
    ids, ref = run(sampler, x, hs, params, u)
    assert check(ids, ref, f"wide top-k {dtype}") <= 6


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_wide_nucleus_rows(sampler, dtype):
    """Top-p only, nuclei of a few hundred to a few thousand values (one block
    per row): the bin-count pass and the key pass, with ties straddling the
    candidate set's last bin, penalised history columns inside the nucleus,
    negative temperatures; nuclei past the key capacity take the multi-pass
    path."""
    B, V = 160, 151936
    x = make_logits(81, B, V, 3.0, dtype=torch.float32)
    top = x.max(dim=1).values
    for b in range(0, B, 10):       # a plateau of ~1500 equal values a few nats below the max
        x[b, b % 7::97] = top[b] - 3.0 - 0.01 * (b % 13)
    for b in range(3, B, 10):       # a narrow band of near-equal values
        x[b, 5000:5600] = top[b] - 2.0 + torch.arange(600, dtype=torch.float32) * 1e-4
    x = x.to(dtype)
    hs = make_histories(82, B, V, 512)
    for b in range(3, B, 10):       # history ids inside the band
        hs[b] = hs[b] + list(range(5000, 5600, 7))
    rng = np.random.default_rng(83)
    params = []
    for b in range(B):
        pen = dict(repetition_penalty=1.1, presence_penalty=0.3, frequency_penalty=0.1) if b % 2 else {}
        params.append(SamplingParams(temperature=float(rng.choice([0.5, 0.7, 1.0, -0.8, 1.3])),
                                     top_k=-1, top_p=float(rng.choice([0.6, 0.8, 0.9, 0.95, 0.99])), **pen))
    u = make_uniforms(84, B)
    ids, ref = run(sampler, x, hs, params, u)
    assert check(ids, ref, f"wide nucleus {dtype}") <= 8


def test_philox_default_stream_matches_oracle(sampler):
    from b200_sampler import B200Sampler
    s = B200Sampler(seed=99)
    B, V = 16, 3000
    x = make_logits(11, B, V)
    params = [SamplingParams(temperature=1.0, top_k=100)] * B
    for call in range(3):
        got = s.select_batch(x.cuda(), [[]] * B, params)
        u = O.philox_uniforms(99, call, B)
        ref = O.sample_batch(x.numpy(), [[]] * B, params, uniforms=u)
        check(got, ref, f"philox call {call}")


def test_errors_match_reference_behaviour(sampler):
    V = 64
    x = torch.zeros(3, V)
    x[0, 5] = float("nan")
    x[1, 7] = float("inf")
    x[2] = float("-inf")
    p = SamplingParams(temperature=1.0, top_k=4)
    for r in range(3):
        with pytest.raises(RuntimeError):
            sampler.select(x[r], [], p)
    # greedy: NaN is the max, first index wins
    g = SamplingParams(temperature=0.0)
    assert sampler.select(x[0], [], g) == 5
    with pytest.raises(IndexError):
        sampler.select(torch.zeros(V), [V + 3], SamplingParams(temperature=0.0, repetition_penalty=1.3))


def test_deterministic(sampler):
    from b200_sampler.workloads import headline
    w = headline(batch=32)
    xd = w.logits.cuda()
    a = sampler.select_batch(xd, w.histories, w.params, uniforms=w.uniforms)
    b = sampler.select_batch(xd, w.histories, w.params, uniforms=w.uniforms)
    assert a == b


def test_logits_not_modified(sampler):
    x = make_logits(5, 4, 1000).cuda()
    before = x.clone()
    sampler.select_batch(x, [[1, 2, 3]] * 4, [SamplingParams(temperature=0.0, repetition_penalty=2.0)] * 4)
    assert torch.equal(x, before)
