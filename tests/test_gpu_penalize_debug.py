"""Debug readback of the penalised logits (``ns_penalize_debug``), bit-exact
against the oracle's restatement of the reference's penalty step
(``sampling/sampler.py:93-108`` plus the frequency / presence extension)."""
import numpy as np
import pytest
import torch

from oracle import sampler_oracle as O
from b200_sampler.params import SamplingParams
from b200_sampler.workloads import make_histories, make_logits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sampler():
    from b200_sampler import B200Sampler
    return B200Sampler(seed=3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_penalised_logits_bit_exact(sampler, dtype):
    B, V = 12, 151936
    x = make_logits(500, B, V, 3.0).to(dtype)
    hs = make_histories(501, B, V, 700, dist="zipf")          # many repeats
    hs[3] = []                                                 # no history
    hs[4] = hs[4] * 7                                          # 4900 ids, > one staging chunk
    rng = np.random.default_rng(502)
    params = [SamplingParams(temperature=0.7, repetition_penalty=float(rng.choice([1.0, 1.1, 0.8, 1.5])),
                             presence_penalty=float(rng.choice([0.0, 0.5, -0.25])),
                             frequency_penalty=float(rng.choice([0.0, 0.3, 0.01])))
              for _ in range(B)]
    params[5] = SamplingParams(temperature=0.7)               # neutral penalties: the widened row
    got = sampler.penalized_logits(x.cuda(), hs, params).cpu().numpy()
    xf = x.float().numpy()
    for b in range(B):
        p = params[b]
        want = O.penalize_row(xf[b], hs[b], p.repetition_penalty, p.presence_penalty, p.frequency_penalty)
        assert np.array_equal(got[b].view(np.uint32), want.view(np.uint32)), b


def test_out_of_range_history_id_raises(sampler):
    x = make_logits(510, 2, 1000, 1.0)
    with pytest.raises(IndexError):
        sampler.penalized_logits(x.cuda(), [[1, 2], [5, 1000]], [SamplingParams(repetition_penalty=1.2)] * 2)
