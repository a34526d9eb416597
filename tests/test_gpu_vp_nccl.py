"""Vocab-parallel sampling across real GPUs: one process per GPU over NCCL.

Each rank holds a column slice of every row; ``VocabParallelSampler`` must
return, on every rank, the ids ``B200Sampler`` returns on the whole rows.
Skipped when fewer than two GPUs are visible.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errq):
    try:
        import torch.distributed as dist
        from b200_sampler import B200Sampler, VocabParallelSampler
        from b200_sampler.params import SamplingParams
        from b200_sampler.workloads import make_histories, make_logits, make_uniforms
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        B, V = 40, 151936
        x = make_logits(51, B, V, 3.0, spike_frac=0.01)
        hs = make_histories(52, B, V, 300)
        rng = np.random.default_rng(53)
        params = []
        for b in range(B):
            if b % 7 == 0:
                params.append(SamplingParams(temperature=0.0, repetition_penalty=1.2, frequency_penalty=0.3))
            elif b % 7 == 3:
                params.append(SamplingParams(temperature=0.9, top_k=-1, top_p=0.85))   # gathered-rows path
            else:
                params.append(SamplingParams(temperature=float(rng.choice([0.7, 1.2])),
                                             top_k=int(rng.choice([10, 50, 100])), top_p=0.9,
                                             repetition_penalty=1.1, presence_penalty=0.5))
        u = make_uniforms(54, B)
        w = (V + world - 1) // world
        off = rank * w
        width = min(w, V - off)
        vps = VocabParallelSampler(V, off, width, seed=9)
        got = vps.select_batch(x[:, off:off + width].to(dev), hs, params, uniforms=u.to(dev))
        ref = B200Sampler(seed=9).select_batch(x.to(dev), hs, params, uniforms=u.to(dev))
        assert got == ref, (rank, [(b, g, r) for b, (g, r) in enumerate(zip(got, ref)) if g != r][:5])
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_vocab_parallel_nccl():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    world = min(n, 8)
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
