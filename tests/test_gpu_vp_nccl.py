"""Vocab-parallel sampling across real GPUs: one process per GPU.

Each rank holds a column slice of every row; ``VocabParallelSampler`` must
return, on every rank, the ids ``B200Sampler`` returns on the whole rows, over
several consecutive steps (the peer exchange alternates its two record
buffers), with the records read in place over NVLink (``peer``) or
all-gathered (``gather``).  A one-rank group runs the peer path (flags,
epochs, record parity) on a single GPU.
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


def _worker(rank, world, port, errq, transports=("peer", "gather"), steps=3):
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
        w = (V + world - 1) // world
        off = rank * w
        width = min(w, V - off)
        xs = x[:, off:off + width].to(dev)
        ref_sampler = B200Sampler(seed=9)
        for transport in transports:
            vps = VocabParallelSampler(V, off, width, seed=9, transport=transport)
            assert vps.transport == transport
            for step in range(steps):
                u = make_uniforms(54 + step, B)
                if step == 2:   # larger records: the peer buffers grow collectively
                    ps = [SamplingParams(temperature=0.8, top_k=200, top_p=0.95, repetition_penalty=1.1)
                          for _ in range(B)]
                else:
                    ps = params
                got = vps.select_batch(xs, hs, ps, uniforms=u.to(dev))
                ref = ref_sampler.select_batch(x.to(dev), hs, ps, uniforms=u.to(dev))
                assert got == ref, (rank, transport, step,
                                    [(b, g, r) for b, (g, r) in enumerate(zip(got, ref)) if g != r][:5])
            vps.close()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def _spawn(world, **kw):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errq), kwargs=kw) for r in range(world)]
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


def test_vocab_parallel_one_rank_peer():
    _spawn(1, transports=("peer",), steps=4)


def test_vocab_parallel_nccl():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    _spawn(min(n, 8))
