"""Host side of the vocab-parallel mode, world size 2 over gloo on CPU.

Two spawned ranks check (1) ``gather_records`` returns every rank's record in
rank order, (2) ``gather_full_rows`` rebuilds whole rows from slices of
unequal width, and (3) the exchange protocol itself: each rank keeps only its
slice's top-k candidates (ties at the k-th scaled value kept) -- a numpy
restatement of what ``ns_vp_local`` writes -- the candidates are exchanged
with ``gather_records``, and sampling the row rebuilt from the union gives the
oracle's id for the whole row.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

V = 5003
B = 12
BOUNDS = [(0, 2001), (2001, V - 2001)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _params():
    from b200_sampler.params import SamplingParams
    rng = np.random.default_rng(3)
    ps = []
    for b in range(B):
        if b % 4 == 0:
            ps.append(SamplingParams(temperature=0.0, repetition_penalty=1.3, frequency_penalty=0.2))
        else:
            ps.append(SamplingParams(temperature=float(rng.choice([0.6, 1.0, -0.9])), top_k=int(rng.choice([3, 17, 64])),
                                     top_p=float(rng.choice([1.0, 0.8])), repetition_penalty=1.1,
                                     presence_penalty=0.4, frequency_penalty=0.1))
    return ps


def _inputs():
    from b200_sampler.workloads import make_histories, make_logits, make_uniforms
    x = make_logits(8, B, V, 2.0).numpy()
    x[5, 1990:2020] = 9.0                  # a tie group across the slice boundary
    return x, make_histories(9, B, V, 150), make_uniforms(10, B).numpy()


def _local_candidates(xrow, hist, p, off, w):
    """Slice's candidates as (penalised x, global id): greedy -> its first
    argmax; sampled -> every value whose scaled value reaches the slice's k-th."""
    from oracle import sampler_oracle as O
    hl = [h - off for h in hist if off <= h < off + w]
    xp = O.penalize_row(xrow[off:off + w], hl, p.repetition_penalty, p.presence_penalty, p.frequency_penalty)
    T = np.float32(p.temperature)
    if T == 0:
        j = O.greedy_argmax(xp)
        return [(float(xp[j]), off + j)]
    y = (xp / T).astype(np.float32)
    fin = np.isfinite(y)
    if fin.sum() <= p.top_k:
        keep = fin
    else:
        thr = np.sort(y[fin])[::-1][p.top_k - 1]
        keep = fin & (y >= thr)
    return [(float(xp[j]), off + int(j)) for j in np.nonzero(keep)[0]]


def _worker(rank, world, port, errq):
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from b200_sampler.vocab_parallel import gather_full_rows, gather_records
        from oracle import sampler_oracle as O

        # (1) records in rank order
        rec = torch.arange(7, dtype=torch.int64) + 100 * rank
        g = gather_records(rec).view(world, 7)
        assert torch.equal(g[0], torch.arange(7)) and torch.equal(g[1], torch.arange(7) + 100)

        x, hs, u = _inputs()
        off, w = BOUNDS[rank]
        # (2) whole rows back from unequal slices
        full = gather_full_rows(torch.from_numpy(x[:, off:off + w].copy()), [b[0] for b in BOUNDS],
                                [b[1] for b in BOUNDS], V)
        assert torch.equal(full, torch.from_numpy(x))

        # (3) the protocol: candidates per slice, exchanged, sampled from the union
        params = _params()
        cap = 96
        recs = np.zeros((B, cap, 2), dtype=np.float64)   # (x, id); count in a side array
        counts = np.zeros(B, dtype=np.int64)
        for b in range(B):
            c = _local_candidates(x[b], hs[b], params[b], off, w)
            assert len(c) <= cap
            counts[b] = len(c)
            recs[b, :len(c)] = c
        flat = torch.cat([torch.from_numpy(counts).double(), torch.from_numpy(recs).reshape(-1)])
        allr = gather_records(flat).view(world, -1).numpy()
        for b in range(B):
            # columns outside the union get the value whose scaled logit is -inf
            fill = np.inf if np.float32(params[b].temperature) < 0 else -np.inf
            xr = np.full(V, fill, dtype=np.float32)
            for r in range(world):
                n = int(allr[r, b])
                ent = allr[r, B:].reshape(B, cap, 2)[b, :n]
                xr[ent[:, 1].astype(np.int64)] = ent[:, 0].astype(np.float32)
            p = params[b]
            from b200_sampler.params import SamplingParams
            nopen = SamplingParams(temperature=p.temperature, top_k=p.top_k, top_p=p.top_p)
            got = O.sample_row(xr, [], nopen, float(u[b]))
            ref = O.sample_row(x[b], hs[b], p, float(u[b]))
            assert got.token == ref.token, (rank, b, got.token, ref.token)
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent, which fails the test
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_vocab_parallel_host_protocol_gloo_world2():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
