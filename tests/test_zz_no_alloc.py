"""ns_sample_noalloc: sampling for callers that may not allocate device memory.

Some engines hand every byte of device memory to their own pool at start-up,
and some plug-ins run inside a host runtime that owns all allocation; neither
can cudaMalloc a workspace for a sampling step.  ns_sample_noalloc takes no
workspace and puts the long-history scratch in a fixed array built into the
library.  These tests call it through the C ABI on histories long enough to
need that scratch, two calls in a row with different inputs, and require the
same ids as ns_sample with a caller workspace (both run the same kernel, so
the ids must be identical).  A size beyond the array is refused.

Kept in a file that pytest collects last.
"""
import numpy as np
import pytest
import torch

from b200_sampler import _lib
from b200_sampler.params import SamplingParams, pack_params
from b200_sampler.workloads import make_logits, make_uniforms

pytestmark = pytest.mark.gpu

V = 151936
DTYPES = {torch.float32: _lib.NS_DTYPE_F32, torch.bfloat16: _lib.NS_DTYPE_BF16}


def _inputs(seed, B, H, dtype, dev):
    """Logits, CSR histories of H ids per row (mostly distinct: more than a
    block's shared memory keeps), packed params and uniforms."""
    rng = np.random.default_rng(seed)
    x = make_logits(seed, B, V, 3.0).to(dtype).to(dev)
    hist = rng.integers(0, V, size=B * H).astype(np.int32)
    offs = np.arange(0, B * H + 1, H, dtype=np.int64)
    params = []
    for b in range(B):
        pen = dict(repetition_penalty=[1.1, 1.3, 0.9][b % 3], presence_penalty=[0.0, 0.5][b % 2],
                   frequency_penalty=[0.0, 0.3, 0.05][b % 3])
        kind = b % 4
        if kind == 0:
            params.append(SamplingParams(temperature=0.0, **pen))
        elif kind == 1:
            params.append(SamplingParams(temperature=0.7, top_k=50, top_p=0.9, **pen))
        elif kind == 2:
            params.append(SamplingParams(temperature=1.0, top_p=0.8, **pen))
        else:
            params.append(SamplingParams(temperature=-0.8, top_k=20, **pen))
    p = torch.from_numpy(pack_params(params)).to(dev)
    u = make_uniforms(seed + 1, B).to(dev)
    return x, torch.from_numpy(hist).to(dev), torch.from_numpy(offs).to(dev), p, u


def _args(x, hist, offs, H, p, u, out):
    B = x.shape[0]
    pp = p.data_ptr()
    return [x.data_ptr(), DTYPES[x.dtype], B, V, x.stride(0), hist.data_ptr(), offs.data_ptr(), H,
            pp, pp + 4 * B, pp + 8 * B, pp + 12 * B, pp + 16 * B, pp + 20 * B,
            u.data_ptr(), 11, 0, out.data_ptr()]


def _with_workspace(lib, x, hist, offs, H, p, u, stream):
    B = x.shape[0]
    out = torch.full((B,), -100, dtype=torch.int64, device=x.device)
    need = _lib.workspace_bytes(B, V, H)
    ws = torch.empty(need + 256, dtype=torch.uint8, device=x.device)
    base = (ws.data_ptr() + 255) // 256 * 256
    rc = lib.ns_sample(*_args(x, hist, offs, H, p, u, out), base, need, stream)
    assert rc == _lib.NS_OK, _lib.status_string(rc)
    torch.cuda.synchronize()
    return out.cpu().tolist()


def test_noalloc_matches_the_workspace_call_two_calls_in_a_row():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    # (rows, history ids per row, dtype): 160 rows run one block per row, 8
    # rows run 8-block clusters, so the two calls lay out the scratch
    # differently; both need scratch, and within the array's limit
    cases = [(160, 4096, torch.float32, 501), (8, 16384, torch.bfloat16, 502)]
    for B, H, dtype, seed in cases:
        need = _lib.workspace_bytes(B, V, H)
        assert 0 < need <= _lib.NS_NOALLOC_SCRATCH_BYTES, (B, H, need)
    results = []
    for B, H, dtype, seed in cases:
        x, hist, offs, p, u = _inputs(seed, B, H, dtype, dev)
        out = torch.full((B,), -100, dtype=torch.int64, device=dev)
        rc = lib.ns_sample_noalloc(*_args(x, hist, offs, H, p, u, out), stream)
        assert rc == _lib.NS_OK, _lib.status_string(rc)
        torch.cuda.synchronize()
        results.append((out.cpu().tolist(), (x, hist, offs, H, p, u)))
    for got, (x, hist, offs, H, p, u) in results:
        want = _with_workspace(lib, x, hist, offs, H, p, u, stream)
        assert min(got) >= 0, got
        assert got == want


def test_noalloc_refuses_sizes_beyond_its_scratch():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, H = 256, 32768
    assert _lib.workspace_bytes(B, V, H) > _lib.NS_NOALLOC_SCRATCH_BYTES
    out = torch.full((B,), -100, dtype=torch.int64, device=dev)
    big = torch.empty((B, V), dtype=torch.float32, device=dev)
    hist_big = torch.zeros(B * H, dtype=torch.int32, device=dev)
    offs_big = torch.arange(0, B * H + 1, H, dtype=torch.int64, device=dev)
    pb = torch.from_numpy(pack_params([SamplingParams(temperature=0.7, top_k=50)] * B)).to(dev)
    ub = make_uniforms(504, B).to(dev)
    rc = lib.ns_sample_noalloc(*_args(big, hist_big, offs_big, H, pb, ub, out),
                               torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.NS_ERR_WORKSPACE_TOO_SMALL
    torch.cuda.synchronize()
    assert int(out.max()) == -100 and int(out.min()) == -100     # nothing was launched
