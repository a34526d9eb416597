"""Failure detection on one GPU, in the allowed form: a flag that nothing sets.

The peer merge of the vocab-parallel mode waits (bounded, ~200 ms) until every
rank's flag has reached this rank's step count.  Here both "ranks" live on
this GPU: ``ns_vp_signal`` from rank 0 bumps the step counter and sets rank
0's flag, rank 1's flag is never set.  Every row must report
NS_ERR_DEVICE_TIMEOUT, the kernel must return (the context stays usable), and
once the missing flag is written the same merge must give the ids that
``ns_vp_merge`` gives on the concatenated records.
"""
import ctypes
import time

import pytest
import torch

from b200_sampler import _lib
from b200_sampler.params import SamplingParams, pack_params
from b200_sampler.workloads import make_logits, make_uniforms

pytestmark = pytest.mark.gpu


def _ptrs(values):
    arr = (ctypes.c_void_p * len(values))(*values)
    return ctypes.cast(arr, ctypes.c_void_p), arr


def test_merge_times_out_on_an_unset_flag_and_recovers_once_it_is_set():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    B, V, cap = 32, 151936, 66
    half = V // 2
    bounds = [(0, half), (half, V - half)]
    x = make_logits(41, B, V, 3.0).to(dev)
    params = [SamplingParams(temperature=0.8, top_k=50, top_p=0.95) if b % 4 else SamplingParams(temperature=0.0)
              for b in range(B)]
    p = torch.from_numpy(pack_params(params)).to(dev)
    pp = p.data_ptr()
    u = make_uniforms(42, B).to(dev)
    n = ctypes.c_int64()
    assert lib.ns_vp_record_int64s(B, cap, ctypes.byref(n)) == 0
    recs = torch.empty(2, n.value, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for r, (off, w) in enumerate(bounds):
        view = x[:, off:off + w]
        rc = lib.ns_vp_local(view.data_ptr(), _lib.NS_DTYPE_F32, B, w, int(view.stride(0)), off, V, None, None, 0,
                             pp, pp + 4 * B, pp + 8 * B, None, None, None, cap, recs[r].data_ptr(), None, 0, stream)
        assert rc == 0, _lib.status_string(rc)
    ref = torch.empty(B, dtype=torch.int64, device=dev)
    assert lib.ns_vp_merge(recs.data_ptr(), 2, B, cap, V, pp, pp + 4 * B, pp + 8 * B, u.data_ptr(), 0, 0,
                           ref.data_ptr(), stream) == 0

    # flags of "rank 0" (both entries live here) and its step counter
    words = torch.zeros(3, dtype=torch.int64, device=dev)
    flags, epoch = words[0:2], words[2:3]
    fl_arg, _k1 = _ptrs([flags.data_ptr(), flags.data_ptr()])
    assert lib.ns_vp_signal(fl_arg, 2, 0, epoch.data_ptr(), stream) == 0   # step 1: only flags[0] = 1
    torch.cuda.synchronize()
    assert words.tolist() == [1, 0, 1]

    rec_arg, _k2 = _ptrs([recs[0].data_ptr(), recs[1].data_ptr()])
    out = torch.full((B,), 12345, dtype=torch.int64, device=dev)

    def merge():
        return lib.ns_vp_merge_peers(rec_arg, 2, flags.data_ptr(), epoch.data_ptr(), B, cap, V,
                                     pp, pp + 4 * B, pp + 8 * B, u.data_ptr(), 0, 0, out.data_ptr(), stream)
    t0 = time.monotonic()
    assert merge() == 0
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert out.tolist() == [_lib.NS_ERR_DEVICE_TIMEOUT] * B
    assert 0.1 < waited < 10.0, waited

    # the context is still usable: the late flag arrives, the merge succeeds
    flags[1].fill_(1)
    assert merge() == 0
    torch.cuda.synchronize()
    assert out.tolist() == ref.tolist()
    assert int(out.min()) >= 0
