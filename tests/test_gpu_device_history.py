"""Device-resident histories (ns_hist_append, DeviceHistory).

The reference rebuilds each row's history as prompt + outputs lists on the
host every step (engine/context_builder.py:208-213, outputs appended at
driver/output_processor.py:46).  ns_hist_append keeps it on the device: these
tests check the appended CSR against plain list concatenation, and a decode
loop sampled through DeviceBatch + DeviceHistory (no host lists) against the
same loop through B200Sampler with Python lists: the ids must be identical at
every step.
"""
import numpy as np
import pytest
import torch

from b200_sampler import _lib
from b200_sampler.params import SamplingParams
from b200_sampler.sampler import B200Sampler, DeviceBatch, DeviceHistory
from b200_sampler.workloads import make_logits, make_uniforms

pytestmark = pytest.mark.gpu


def _append_c(ids, offs, new, capacity):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    B = new.numel()
    out_ids = torch.full((capacity,), -7, dtype=torch.int32, device=dev)
    out_offs = torch.full((B + 1,), -7, dtype=torch.int64, device=dev)
    rc = lib.ns_hist_append(None if ids is None else ids.data_ptr(), None if offs is None else offs.data_ptr(), B,
                            new.data_ptr(), out_ids.data_ptr(), out_offs.data_ptr(), capacity,
                            torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.NS_OK, _lib.status_string(rc)
    torch.cuda.synchronize()
    return out_ids.cpu().numpy(), out_offs.cpu().numpy()


def test_hist_append_matches_list_concatenation():
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(11)
    B = 37
    lens = rng.integers(0, 300, size=B)
    lens[5] = 0
    lens[B - 1] = 0
    rows = [rng.integers(0, 151936, size=n).tolist() for n in lens]
    new = rng.integers(0, 151936, size=B)
    new[3] = -6                                   # a failed row's status
    offs = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(lens, out=offs[1:])
    flat = np.concatenate([np.asarray(r, dtype=np.int32) for r in rows])
    total = int(offs[-1])
    out_ids, out_offs = _append_c(torch.from_numpy(flat).to(dev), torch.from_numpy(offs).to(dev),
                                  torch.from_numpy(new.astype(np.int64)).to(dev), total + B + 5)
    want = [r + [int(v) if v >= 0 else -1] for r, v in zip(rows, new)]
    assert out_offs.tolist() == list(np.cumsum([0] + [len(w) for w in want]))
    for b in range(B):
        assert out_ids[out_offs[b]:out_offs[b + 1]].tolist() == want[b]
    assert (out_ids[total + B:] == -7).all()       # nothing past the CSR


def test_hist_append_from_empty_histories_and_capacity_bound():
    dev = torch.device("cuda", 0)
    new = torch.arange(10, 18, dtype=torch.int64, device=dev)
    out_ids, out_offs = _append_c(None, None, new, 8)
    assert out_offs.tolist() == list(range(9))
    assert out_ids.tolist() == list(range(10, 18))
    # a capacity below the result drops the writes past it (no stray writes)
    ids = torch.arange(0, 16, dtype=torch.int32, device=dev)
    offs = torch.tensor([0, 8, 16], dtype=torch.int64, device=dev)
    out_ids, out_offs = _append_c(ids, offs, torch.tensor([100, 200], dtype=torch.int64, device=dev), 12)
    assert out_offs.tolist() == [0, 9, 18]
    assert out_ids.tolist() == list(range(8)) + [100] + list(range(8, 11))


def test_decode_loop_on_device_histories_matches_host_lists():
    """20 decode steps at B=64 with penalties (the history matters every
    step): DeviceBatch + DeviceHistory against B200Sampler on Python lists,
    the same logits and uniforms per step."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, V, steps = 64, 151936, 20
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, V, size=int(rng.integers(1, 200))).tolist() for _ in range(B)]
    params = [SamplingParams(temperature=0.7, top_k=20, top_p=0.8, repetition_penalty=1.3,
                             presence_penalty=0.5, frequency_penalty=0.3) if b % 4 else
              SamplingParams(temperature=0.0, repetition_penalty=1.2, presence_penalty=0.5)
              for b in range(B)]
    host_hist = [list(p) for p in prompts]
    sampler = B200Sampler(seed=3)
    dh = DeviceHistory(prompts, dev, reserve_steps=8)       # grows once on the way
    db = DeviceBatch(None, params, dev, uniforms=torch.zeros(B), history=dh)
    out = torch.empty(B, dtype=torch.int64, device=dev)
    for t in range(steps):
        # logits that favour recently sampled ids, so the penalties decide often
        x = make_logits(400 + t, B, V, 3.0)
        for b in range(B):
            x[b, host_hist[b][-8:]] += 4.0
        x = x.to(dev)
        u = make_uniforms(500 + t, B)
        want = sampler.select_batch_tensor(x, host_hist, params, uniforms=u.to(dev)).cpu().tolist()
        db.uniforms.copy_(u.to(dev))
        assert db.launch(x, out) == _lib.NS_OK
        dh.append(out)
        got = out.cpu().tolist()
        assert got == want, t
        assert min(got) >= 0
        for b in range(B):
            host_hist[b].append(want[b])
    assert dh.to_lists() == host_hist
    assert dh.max_history == max(len(p) for p in prompts) + steps
