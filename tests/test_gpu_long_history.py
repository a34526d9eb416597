"""Long histories: shared memory does not grow with the history length.

A block keeps at most 1024 distinct history ids in shared memory; a block
whose columns hold more moves its rank arrays (count, column, penalised value
per distinct id) to the caller's workspace.  These tests run histories of
1K-32K ids with heavy duplicates (a few hundred distinct ids: shared memory)
and with mostly distinct ids (the workspace), on one block per row (160 rows)
and on 8-block clusters (8 rows), fp32 and bf16, against the CPU oracle
(reference: sampler.py:93-108 for the penalties, then the sampling chain).
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import sampler_oracle as O
from b200_sampler import _lib
from b200_sampler.params import SamplingParams
from b200_sampler.workloads import make_logits, make_uniforms

pytestmark = pytest.mark.gpu

V = 151936


@pytest.fixture(scope="module")
def sampler():
    from b200_sampler import B200Sampler
    return B200Sampler(seed=99)


def _histories(seed, B, lengths, pool_sizes):
    """Row b: lengths[b % len] ids drawn from a pool of pool_sizes[b % len]
    distinct ids (None: uniform over the vocabulary)."""
    rng = np.random.default_rng(seed)
    hs = []
    for b in range(B):
        n = lengths[b % len(lengths)]
        pool = pool_sizes[b % len(pool_sizes)]
        if pool is None:
            h = rng.integers(0, V, size=n)
        else:
            ids = rng.choice(V, size=pool, replace=False)
            h = ids[rng.integers(0, pool, size=n)]
        hs.append([int(i) for i in h])
    return hs


def _params(seed, B):
    rng = np.random.default_rng(seed)
    out = []
    for b in range(B):
        kind = b % 5
        pen = dict(repetition_penalty=float(rng.choice([1.1, 1.3, 0.9])),
                   presence_penalty=float(rng.choice([0.0, 0.5])),
                   frequency_penalty=float(rng.choice([0.0, 0.3, 0.05])))
        if kind == 0:
            out.append(SamplingParams(temperature=0.0, **pen))
        elif kind == 1:
            out.append(SamplingParams(temperature=0.7, top_k=50, top_p=0.9, **pen))
        elif kind == 2:
            out.append(SamplingParams(temperature=-0.8, top_k=20, **pen))
        elif kind == 3:
            out.append(SamplingParams(temperature=1.0, top_p=0.8, **pen))
        else:
            out.append(SamplingParams(temperature=1.3, top_k=300, top_p=0.95, **pen))
    return out


def _check(ids, ref, ctx, max_exempt):
    n_exempt = 0
    for b, r in enumerate(ref):
        assert not r.error, (ctx, b, r.error)
        if ids[b] != r.token:
            assert r.exempt and ids[b] in r.allowed, (ctx, b, ids[b], r.token, r.exempt)
            n_exempt += 1
    assert n_exempt <= max_exempt, (ctx, n_exempt)


@pytest.mark.parametrize("H", [1024, 4096, 16384, 32768])
@pytest.mark.parametrize("B", [160, 8])
def test_long_history_parity(sampler, H, B):
    """Half the rows draw H ids from a few hundred distinct ids, half from the
    whole vocabulary (up to ~H distinct ids per row)."""
    dtype = torch.float32 if H in (1024, 16384) else torch.bfloat16
    x = make_logits(300 + H, B, V, 3.0).to(dtype)
    hs = _histories(301 + H, B, [H, H // 2 + 7], [300, None, 60, None])
    params = _params(302 + H, B)
    u = make_uniforms(303 + H, B)
    ids = sampler.select_batch_tensor(x.cuda(), hs, params, uniforms=u.cuda()).cpu().tolist()
    ref = O.sample_batch(x.float().numpy(), hs, params, uniforms=u.numpy())
    _check(ids, ref, f"B {B} H {H} {dtype}", max_exempt=2)


def test_distinct_ids_at_the_shared_memory_limit(sampler):
    """Rows with 1023, 1024 and 1025 distinct ids on one block per row: the
    last one is the first that moves to the workspace."""
    B = 150
    x = make_logits(320, B, V, 3.0)
    rng = np.random.default_rng(321)
    hs = []
    for b in range(B):
        d = 1023 + b % 3
        ids = rng.choice(V, size=d, replace=False)
        h = np.concatenate([ids, ids[rng.integers(0, d, size=2000 - d)]])
        rng.shuffle(h)
        hs.append([int(i) for i in h])
    params = _params(322, B)
    u = make_uniforms(323, B)
    ids = sampler.select_batch_tensor(x.cuda(), hs, params, uniforms=u.cuda()).cpu().tolist()
    ref = O.sample_batch(x.numpy(), hs, params, uniforms=u.numpy())
    _check(ids, ref, "1023..1025 distinct", max_exempt=2)


def test_long_history_needs_the_workspace():
    """A history longer than 1024 ids with no (or too small a) workspace is
    refused before any launch; with the queried size it runs."""
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    B, H = 4, 2048
    x = make_logits(330, B, V, 3.0).to(dev)
    hist = torch.randint(0, V, (B * H,), dtype=torch.int32, device=dev)
    offs = torch.arange(0, B * H + 1, H, dtype=torch.int64, device=dev)
    T = torch.full((B,), 0.7, device=dev)
    k = torch.full((B,), 50, dtype=torch.int32, device=dev)
    p = torch.full((B,), 0.9, device=dev)
    rp = torch.full((B,), 1.2, device=dev)
    out = torch.empty(B, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def call(ws, nbytes):
        return lib.ns_sample(x.data_ptr(), _lib.NS_DTYPE_F32, B, V, V, hist.data_ptr(), offs.data_ptr(), H,
                             T.data_ptr(), k.data_ptr(), p.data_ptr(), rp.data_ptr(), None, None,
                             None, 7, 0, out.data_ptr(), ws, nbytes, stream)

    need = _lib.workspace_bytes(B, V, H)
    assert need >= B * 12 * H
    assert call(None, 0) == _lib.NS_ERR_WORKSPACE_TOO_SMALL
    ws = torch.empty(need + 512, dtype=torch.uint8, device=dev)
    base = (ws.data_ptr() + 255) // 256 * 256
    assert call(base, need - 1) == _lib.NS_ERR_WORKSPACE_TOO_SMALL
    assert call(base + 16, need) == _lib.NS_ERR_WORKSPACE_TOO_SMALL      # not 256-byte aligned
    assert call(base, need) == _lib.NS_OK
    torch.cuda.synchronize()
    assert int(out.min()) >= 0
