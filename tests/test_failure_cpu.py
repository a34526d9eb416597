"""Failure detection on the host, without a GPU.

(1) A world-size-2 gloo group in which rank 1 joins but never calls the
    record exchange: rank 0's ``gather_records`` must end with an error within
    the process group's short timeout instead of waiting for good.
(2) The vocab-parallel sampler's recovery after the merge kernel's bounded
    flag wait gave up: fakes stand in for the device flags and the merge.
    A late peer (its flag arrives while the host waits) costs one more merge;
    a peer that never signals makes the call raise and the sampler refuse
    every later call.
"""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from b200_sampler import _lib


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _silent_peer_worker(rank, world, port, resq):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    from b200_sampler.vocab_parallel import gather_records
    if rank == 0:
        t0 = time.monotonic()
        try:
            gather_records(torch.arange(4, dtype=torch.int64))
            resq.put(("no error", time.monotonic() - t0))
        except Exception as e:  # the expected outcome
            resq.put((type(e).__name__, time.monotonic() - t0))
    else:
        # joined the group, never calls the exchange; leaves once rank 0 is done
        deadline = time.monotonic() + 60
        while resq.empty() and time.monotonic() < deadline:
            time.sleep(0.05)
    os._exit(0)   # no destroy_process_group: it would wait for the silent peer


def test_exchange_with_a_silent_rank_times_out():
    ctx = mp.get_context("spawn")
    resq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_silent_peer_worker, args=(r, 2, port, resq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish"
    assert not resq.empty(), "rank 0 reported nothing"
    what, waited = resq.get()
    assert what != "no error", "the exchange completed without its peer"
    assert waited < 30.0, waited        # bounded by the 3 s group timeout, not unbounded


def test_wait_for_peers_sees_a_late_flag_and_gives_up_on_a_missing_one():
    from b200_sampler.vocab_parallel import wait_for_peers
    calls = {"n": 0}

    def late():
        calls["n"] += 1
        return ([5, 5 if calls["n"] >= 4 else 4], 5)
    assert wait_for_peers(late, timeout_s=5.0, poll_s=0.001)
    assert calls["n"] == 4
    t0 = time.monotonic()
    assert not wait_for_peers(lambda: ([5, 4], 5), timeout_s=0.2, poll_s=0.01)
    assert 0.15 < time.monotonic() - t0 < 2.0


class _FakeExchange:
    def __init__(self, flags_after):
        self.reads = 0
        self.flags_after = flags_after   # reads before the late flag appears (None: never)

    def read_state(self, stream):
        self.reads += 1
        ok = self.flags_after is not None and self.reads > self.flags_after
        return [3, 3 if ok else 2], 3


class _Stream:
    def synchronize(self):
        pass


def _sampler():
    from b200_sampler.vocab_parallel import VocabParallelSampler
    s = VocabParallelSampler.__new__(VocabParallelSampler)   # no process group needed for this path
    s._broken = None
    s.peer_wait_s = 0.3
    return s


def test_timeout_recovery_merges_again_once_the_late_flag_arrives():
    s = _sampler()
    out = torch.full((4,), _lib.NS_ERR_DEVICE_TIMEOUT, dtype=torch.int64)
    merges = {"n": 0}

    def merge():
        merges["n"] += 1
        out.copy_(torch.tensor([7, 8, 9, 10]))
        return _lib.NS_OK
    rc = s._recover_timeout(_FakeExchange(flags_after=3), _Stream(), merge, out)
    assert rc == _lib.NS_OK and merges["n"] == 1
    assert out.tolist() == [7, 8, 9, 10]
    assert s._broken is None


def test_timeout_recovery_poisons_the_sampler_when_a_peer_never_signals():
    s = _sampler()
    out = torch.full((4,), _lib.NS_ERR_DEVICE_TIMEOUT, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="did not signal"):
        s._recover_timeout(_FakeExchange(flags_after=None), _Stream(), lambda: _lib.NS_OK, out)
    assert s._broken is not None and "[1]" in s._broken
    # every later call refuses before touching a device
    from b200_sampler.params import SamplingParams
    with pytest.raises(RuntimeError, match="unusable"):
        s._run(torch.zeros(1, 1), None, [SamplingParams()], None, None, retry=True)


def test_timeout_recovery_poisons_when_the_second_merge_times_out_too():
    s = _sampler()
    out = torch.full((2,), _lib.NS_ERR_DEVICE_TIMEOUT, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="again"):
        s._recover_timeout(_FakeExchange(flags_after=0), _Stream(), lambda: _lib.NS_OK, out)
    assert s._broken is not None
