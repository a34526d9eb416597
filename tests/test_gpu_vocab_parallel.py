"""Vocab-parallel sampling through the C ABI, on one GPU.

The n ranks are emulated: ``ns_vp_local`` runs once per column slice, the
records are concatenated in rank order (what the all-gather produces) and
``ns_vp_merge`` samples from them.  The ids must equal ``ns_sample`` on the
whole rows with the same uniforms -- exactly, since the merge sees the same
survivors in the same order -- and the CPU oracle's.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import sampler_oracle as O
from b200_sampler import _lib
from b200_sampler.params import SamplingParams, pack_params
from b200_sampler.workloads import make_histories, make_logits, make_uniforms

pytestmark = pytest.mark.gpu

_DT = {torch.float32: _lib.NS_DTYPE_F32, torch.bfloat16: _lib.NS_DTYPE_BF16, torch.float16: _lib.NS_DTYPE_F16}


def _csr(hs, dev):
    lens = np.array([len(h) for h in hs], dtype=np.int64)
    offs = np.zeros(len(hs) + 1, dtype=np.int64)
    np.cumsum(lens, out=offs[1:])
    flat = np.concatenate([np.asarray(h, dtype=np.int32) for h in hs]) if lens.sum() else np.zeros(1, np.int32)
    return (torch.from_numpy(flat).to(dev), torch.from_numpy(offs).to(dev), int(lens.max()) if len(hs) else 0)


def vp_sample(x_dev, hs, params, u_dev, bounds, cap):
    """Emulated ranks: local step per slice, concatenated records, merge."""
    lib = _lib.load()
    B, V = x_dev.shape
    dev = x_dev.device
    p = torch.from_numpy(pack_params(params)).to(dev)
    pp = p.data_ptr()
    hid, hoff, hmax = _csr(hs, dev)
    n = ctypes.c_int64()
    assert lib.ns_vp_record_int64s(B, cap, ctypes.byref(n)) == 0
    recs = torch.empty(len(bounds), n.value, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    ws_bytes = max(_lib.workspace_bytes(B, w, hmax) for _, w in bounds)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)   # the slices run one after another
    for r, (off, w) in enumerate(bounds):
        view = x_dev[:, off:off + w]
        rc = lib.ns_vp_local(view.data_ptr(), _DT[x_dev.dtype], B, w, int(view.stride(0)), off, V,
                             hid.data_ptr(), hoff.data_ptr(), hmax,
                             pp, pp + 4 * B, pp + 8 * B, pp + 12 * B, pp + 16 * B, pp + 20 * B,
                             cap, recs[r].data_ptr(), ws.data_ptr(), ws_bytes, stream)
        assert rc == 0, _lib.status_string(rc)
    out = torch.empty(B, dtype=torch.int64, device=dev)
    rc = lib.ns_vp_merge(recs.data_ptr(), len(bounds), B, cap, V, pp, pp + 4 * B, pp + 8 * B,
                         None if u_dev is None else u_dev.data_ptr(), 7, 3, out.data_ptr(), stream)
    assert rc == 0, _lib.status_string(rc)
    return out.cpu().tolist(), recs


def whole_rows(x_dev, hs, params, u_dev):
    from b200_sampler import B200Sampler
    s = B200Sampler(seed=7)
    s.offset = 3
    return s.select_batch_tensor(x_dev, hs, params, uniforms=u_dev).cpu().tolist()


def even(V, n):
    w = (V + n - 1) // n
    return [(r * w, min(w, V - r * w)) for r in range(n)]


def mixed_params(B, seed):
    rng = np.random.default_rng(seed)
    ps = []
    for b in range(B):
        if b % 5 == 0:
            ps.append(SamplingParams(temperature=0.0, repetition_penalty=1.2, presence_penalty=0.5,
                                     frequency_penalty=0.3))
        else:
            ps.append(SamplingParams(temperature=float(rng.choice([0.7, 1.3, -0.8])),
                                     top_k=int(rng.choice([1, 5, 50, 128])),
                                     top_p=float(rng.choice([1.0, 0.9, 0.5])),
                                     repetition_penalty=float(rng.choice([1.0, 1.1])),
                                     presence_penalty=float(rng.choice([0.0, 0.5])),
                                     frequency_penalty=float(rng.choice([0.0, 0.3]))))
    return ps


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("split", ["even2", "even8", "uneven3"])
def test_vp_matches_whole_rows_and_oracle(dtype, split):
    B, V = 24, 151936
    bounds = {"even2": even(V, 2), "even8": even(V, 8),
              "uneven3": [(0, 50001), (50001, 3), (50004, V - 50004)]}[split]
    x = make_logits(11, B, V, 3.0, spike_frac=0.01, dtype=dtype)
    hs = make_histories(12, B, V, 400)
    params = mixed_params(B, 13)
    u = make_uniforms(14, B)
    xd, ud = x.cuda(), u.cuda()
    got, _ = vp_sample(xd, hs, params, ud, bounds, cap=160)
    assert got == whole_rows(xd, hs, params, ud)
    ref = O.sample_batch(x.float().numpy(), hs, params, uniforms=u.numpy())
    for b, r in enumerate(ref):
        assert got[b] == r.token or (r.exempt and got[b] in r.allowed), (b, got[b], r.token)


def test_vp_config4_eight_slices():
    """Benchmark configuration 4: 128 rows, 8 slices of 18992, k 50, p 0.95, T 0.8."""
    B, V = 128, 151936
    x = make_logits(4, B, V, 3.0)
    params = [SamplingParams(temperature=0.8, top_k=50, top_p=0.95)] * B
    u = make_uniforms(5, B)
    xd, ud = x.cuda(), u.cuda()
    got, recs = vp_sample(xd, [[]] * B, params, ud, even(V, 8), cap=66)
    assert got == whole_rows(xd, [[]] * B, params, ud)
    counts = recs[:, :B].cpu()
    assert int(counts.min()) >= 1 and int(counts.max()) <= 66
    ref = O.sample_batch(x.numpy(), [[]] * B, params, uniforms=u.numpy())
    for b, r in enumerate(ref):
        assert got[b] == r.token or (r.exempt and got[b] in r.allowed), b


def test_vp_philox_default_stream():
    B, V = 16, 32000
    x = make_logits(21, B, V)
    params = [SamplingParams(temperature=1.0, top_k=40, top_p=0.9)] * B
    xd = x.cuda()
    got, _ = vp_sample(xd, [[]] * B, params, None, even(V, 4), cap=64)
    assert got == whole_rows(xd, [[]] * B, params, None)


def test_vp_statuses():
    B, V = 6, 9000
    x = torch.zeros(B, V)
    x[0, 8999] = float("nan")                      # sampled row, NaN in the last slice
    x[1] = float("-inf")                           # nothing finite anywhere
    x[2, 100:140] = 5.0                            # 40 ties in one slice, k 10, cap 16: overflow
    params = [SamplingParams(temperature=1.0, top_k=10),
              SamplingParams(temperature=1.0, top_k=10),
              SamplingParams(temperature=1.0, top_k=10),
              SamplingParams(temperature=1.0, top_k=-1, top_p=0.9),   # top-k off: no candidate record
              SamplingParams(temperature=0.0),
              SamplingParams(temperature=0.0, repetition_penalty=1.5)]
    x[4, 7000] = float("nan")                      # greedy: NaN is the max
    hs = [[], [], [], [], [], [V + 5]]             # bad id on a greedy row
    got, _ = vp_sample(x.cuda(), hs, params, make_uniforms(1, B).cuda(), even(V, 3), cap=16)
    assert got[0] == _lib.NS_ERR_INVALID_DISTRIBUTION
    assert got[1] == _lib.NS_ERR_INVALID_DISTRIBUTION
    assert got[2] == _lib.NS_ERR_CANDIDATE_OVERFLOW
    assert got[3] == _lib.NS_ERR_UNSUPPORTED
    assert got[4] == 7000
    assert got[5] == _lib.NS_ERR_TOKEN_ID_OUT_OF_RANGE


def test_vp_sampler_class_single_rank():
    """VocabParallelSampler with a one-rank gloo group: the whole vocab is one
    slice; top-k-off rows take the gathered-rows path."""
    import os
    import torch.distributed as dist
    from b200_sampler import B200Sampler, VocabParallelSampler
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        B, V = 10, 20000
        x = make_logits(31, B, V).cuda()
        hs = make_histories(32, B, V, 64)
        params = mixed_params(B, 33)
        params[3] = SamplingParams(temperature=0.9, top_k=-1, top_p=0.8)
        u = make_uniforms(34, B).cuda()
        vps = VocabParallelSampler(V, 0, V, seed=5)
        got = vps.select_batch(x, hs, params, uniforms=u)
        assert got == B200Sampler(seed=5).select_batch(x, hs, params, uniforms=u)
    finally:
        dist.destroy_process_group()
