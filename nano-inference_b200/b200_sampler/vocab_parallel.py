"""Vocab-parallel sampling: each rank holds a contiguous column slice of every
row (tensor-parallel lm_head output) and all ranks return the same ids.

No reference counterpart: nano-inference samples whole rows
(``sampling/sampler.py:36-91``).  The steps, per call:

1. ``ns_vp_local`` on this rank's slice: history penalties for the ids the
   slice holds, then per row the slice's top-k survivors (ties at the k-th
   scaled value kept) as 64-bit keys, or one key for greedy rows;
2. the exchange of those fixed-size records (a few KB per row), either
   - ``peer`` (default with NCCL, at most 8 ranks): each rank keeps its record
     in its own device memory, mapped by every other rank (CUDA IPC);
     ``ns_vp_signal`` sets a flag on every rank and ``ns_vp_merge_peers``
     waits for all flags and reads every record in place over NVLink, in the
     merge kernel itself; or
   - ``gather``: ``gather_records``, an all-gather (NCCL or gloo);
3. the merge on every rank: the global top-k with ties, top-p and the
   inverse-CDF draw.  The global top-k set lies inside the union of the
   slices' top-k sets, so the ids equal ``B200Sampler`` on whole rows.

Rows with top-k off or k > 240 have no bounded candidate set; their slices are
all-gathered into whole rows (``gather_full_rows``) and sampled with
``ns_sample`` on every rank.  With ``uniforms=None`` those rows draw from the
Philox stream at their position in that sub-batch (still identical on every
rank).
"""
from __future__ import annotations

import ctypes
import time
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .params import pack_params
from .sampler import _DTYPES, _ROW_ERRORS, B200Sampler
from .workspace import Workspace

FAST_MAX_K = 240       # largest top_k the candidate records serve (kFastK in the kernel)
MAX_CAP = 1024         # record capacity limit (kRankMax in the kernel)
PEER_WAIT_S = 30.0     # host-side wait for late peers after the merge kernel's own ~200 ms bound


def wait_for_peers(read_state: Callable[[], Tuple[Sequence[int], int]], timeout_s: float,
                   poll_s: float = 0.002) -> bool:
    """Poll ``read_state() -> (flags, epoch)`` until every rank's flag has
    reached this rank's step count; False if that does not happen within
    ``timeout_s`` seconds."""
    deadline = time.monotonic() + timeout_s
    while True:
        flags, epoch = read_state()
        if all(int(f) >= int(epoch) for f in flags):
            return True
        if time.monotonic() >= deadline:
            return False
        time.sleep(poll_s)


class _DeviceWords:
    """int64 words of raw device memory, viewed as a tensor (no ownership)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i8", "data": (ptr, False),
                                         "version": 3, "strides": None}


def gather_records(rec: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather equal-length 1-D records; returns [world * len] in rank order."""
    world = dist.get_world_size(group)
    if world == 1:
        return rec.contiguous()
    out = torch.empty(world * rec.numel(), dtype=rec.dtype, device=rec.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, rec.contiguous(), group=group)
    else:
        dist.all_gather(list(out.view(world, -1).unbind(0)), rec.contiguous(), group=group)
    return out


def gather_full_rows(rows: torch.Tensor, offsets: Sequence[int], widths: Sequence[int], vocab_total: int,
                     group=None) -> torch.Tensor:
    """Rebuild whole rows from every rank's slice of the same rows: rows is
    this rank's [n, width_r] slice; returns [n, vocab_total] on every rank."""
    world = dist.get_world_size(group)
    n = rows.shape[0]
    wmax = max(widths)
    pad = torch.zeros(n, wmax, dtype=rows.dtype, device=rows.device)
    pad[:, :rows.shape[1]] = rows
    g = gather_records(pad.reshape(-1), group).view(world, n, wmax)
    full = torch.empty(n, vocab_total, dtype=rows.dtype, device=rows.device)
    for r in range(world):
        full[:, offsets[r]:offsets[r] + widths[r]] = g[r, :, :widths[r]]
    return full


class PeerExchange:
    """Records and flags that every rank of a group reads in place: one device
    buffer per rank (two records, used on alternate steps, then one int64
    flag per rank and this rank's step counter), mapped into every other rank
    with CUDA IPC.  Growing it is collective (every rank calls ``ensure`` with
    the same size)."""

    def __init__(self, lib, group, world: int, rank: int, device: torch.device):
        self.lib, self.group, self.world, self.rank, self.device = lib, group, world, rank, device
        self.rec_bytes = 0
        self.bases: List[int] = []      # rank r's buffer as seen from this process
        self.steps = 0                  # steps exchanged so far (the same on every rank)

    def ensure(self, rec_int64s: int, stream: torch.cuda.Stream):
        need = (rec_int64s * 8 + 255) // 256 * 256
        if need <= self.rec_bytes:
            return
        self.release(stream)
        flag_bytes = ((self.world + 1) * 8 + 255) // 256 * 256   # flags, then the step counter
        with torch.cuda.device(self.device):
            own = ctypes.c_void_p()
            rc = self.lib.ns_vp_peer_alloc(2 * need + flag_bytes, ctypes.byref(own))
            if rc != _lib.NS_OK:
                raise RuntimeError(f"ns_vp_peer_alloc failed: {_lib.status_string(rc)}")
            handle = ctypes.create_string_buffer(_lib.NS_IPC_HANDLE_BYTES)
            rc = self.lib.ns_ipc_handle(own, handle)
            if rc != _lib.NS_OK:
                raise RuntimeError(f"ns_ipc_handle failed: {_lib.status_string(rc)}")
            handles: List[Optional[bytes]] = [handle.raw]
            if self.world > 1:
                handles = [None] * self.world
                dist.all_gather_object(handles, handle.raw, group=self.group)
            bases = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(own.value)
                    continue
                p = ctypes.c_void_p()
                rc = self.lib.ns_ipc_open(ctypes.create_string_buffer(h, len(h)), ctypes.byref(p))
                if rc != _lib.NS_OK:
                    raise RuntimeError(f"ns_ipc_open failed (rank {r}): {_lib.status_string(rc)}")
                bases.append(p.value)
        self.bases, self.rec_bytes = bases, need

    def release(self, stream: torch.cuda.Stream):
        """Collective: once every rank's kernels are done with the buffers,
        unmap the peers' and free this rank's."""
        if not self.bases:
            return
        stream.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for r, b in enumerate(self.bases):
                if r != self.rank:
                    self.lib.ns_ipc_close(ctypes.c_void_p(b))
            self.lib.ns_vp_peer_free(ctypes.c_void_p(self.bases[self.rank]))
        self.bases, self.rec_bytes = [], 0

    def record(self, r: int, parity: int) -> int:
        return self.bases[r] + parity * self.rec_bytes

    def flags(self, r: int) -> int:
        return self.bases[r] + 2 * self.rec_bytes

    def counter(self) -> int:
        """This rank's step counter (device memory, advanced by ns_vp_signal)."""
        return self.flags(self.rank) + 8 * self.world

    def read_state(self, stream: torch.cuda.Stream) -> Tuple[List[int], int]:
        """(every rank's flag in this rank's buffer, this rank's step count),
        read on the host once `stream`'s work is done."""
        stream.synchronize()
        words = torch.as_tensor(_DeviceWords(self.flags(self.rank), self.world + 1), device=self.device)
        v = words.cpu().tolist()
        return v[:self.world], v[self.world]


def _ptr_array(ptrs: Sequence[int]) -> ctypes.c_void_p:
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    return ctypes.cast(arr, ctypes.c_void_p), arr   # keep arr alive with the pointer


class VocabParallelSampler(B200Sampler):
    """``SamplerBase`` over a vocab-parallel slice.

    Args:
        vocab_total: full vocabulary size.
        vocab_offset, vocab_local: this rank's columns
            ``[vocab_offset, vocab_offset + vocab_local)``.
        group: torch.distributed process group (default: the world).
        seed: Philox key for calls without ``uniforms``; rank 0's value is
            broadcast so every rank draws the same uniforms.
        tie_slack: record entries beyond the batch's largest top_k for values
            tied at a slice's k-th value; a row whose slice overflows is
            retried once with the largest capacity.
        transport: "peer" (records read in place over NVLink by the merge
            kernel), "gather" (all-gather), or "auto": "peer" on an NCCL group
            of at most 8 ranks, else "gather".

    Every rank must call with the same histories, params and uniforms (the
    engine replicates them); the logits are this rank's slice.
    """

    def __init__(self, vocab_total: int, vocab_offset: int, vocab_local: int, group=None, device=None,
                 seed: Optional[int] = None, tie_slack: int = 16, transport: str = "auto"):
        super().__init__(device=device, seed=seed)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.vocab_total = int(vocab_total)
        self.vocab_offset = int(vocab_offset)
        self.vocab_local = int(vocab_local)
        self.tie_slack = int(tie_slack)
        geo: List[Optional[tuple]] = [None] * self.world
        dist.all_gather_object(geo, (self.vocab_offset, self.vocab_local, self.seed), group=group)
        self.offsets = [g[0] for g in geo]
        self.widths = [g[1] for g in geo]
        self.seed = int(geo[0][2])
        cover = sorted(zip(self.offsets, self.widths))
        pos = 0
        for o, w in cover:
            if o != pos or w <= 0:
                raise ValueError("rank slices must tile [0, vocab_total) without gaps or overlaps")
            pos += w
        if pos != self.vocab_total:
            raise ValueError("rank slices must cover the whole vocabulary")
        if transport == "auto":
            transport = "peer" if dist.get_backend(group) == "nccl" and self.world <= 8 else "gather"
        if transport not in ("peer", "gather"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self._exchange: Optional[PeerExchange] = None
        self._broken: Optional[str] = None   # set when a peer never signalled: every later call raises
        self.peer_wait_s = PEER_WAIT_S

    def _recover_timeout(self, ex: PeerExchange, stream: torch.cuda.Stream, merge, out: torch.Tensor) -> int:
        """The merge kernel gave up waiting (~200 ms) for a peer's flag.  Host
        skew (a slow first call, a garbage collection) is not a failure: wait
        on the host, up to ``peer_wait_s``, for every flag to reach this step,
        then merge again.  A peer that never signals makes the exchange
        unusable: this call and every later one raise."""
        if not wait_for_peers(lambda: ex.read_state(stream), self.peer_wait_s):
            flags, epoch = ex.read_state(stream)
            late = [r for r, f in enumerate(flags) if f < epoch]
            self._broken = f"rank(s) {late} did not signal step {epoch} within {self.peer_wait_s:.1f} s"
            raise RuntimeError(f"vocab-parallel exchange timed out: {self._broken}")
        rc = merge()
        if rc == _lib.NS_OK and bool((out == _lib.NS_ERR_DEVICE_TIMEOUT).any()):
            self._broken = "the merge timed out again after every flag was set"
            raise RuntimeError(f"vocab-parallel exchange timed out: {self._broken}")
        return rc

    def close(self):
        """Collective: release the peer-exchange buffers (every rank calls it)."""
        if self._exchange is not None:
            self._exchange.release(torch.cuda.current_stream(self._exchange.device))
            self._exchange = None

    def select_batch_tensor(self, logits: torch.Tensor, all_generated_ids, all_sampling_params, *,
                            uniforms: Optional[torch.Tensor] = None,
                            out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self._run(logits, all_generated_ids, all_sampling_params, uniforms, out, retry=True)

    def _run(self, logits, all_generated_ids, all_sampling_params, uniforms, out, retry: bool,
             cap: Optional[int] = None, offset: Optional[int] = None) -> torch.Tensor:
        if self._broken is not None:
            raise RuntimeError(f"vocab-parallel exchange is unusable: {self._broken}")
        if logits.dim() != 2 or logits.shape[1] != self.vocab_local:
            raise ValueError("expected this rank's [batch, vocab_local] slice")
        if logits.dtype not in _DTYPES:
            raise TypeError(f"unsupported logits dtype {logits.dtype}")
        B = int(logits.shape[0])
        if len(all_sampling_params) != B or (all_generated_ids is not None and len(all_generated_ids) != B):
            raise AssertionError("batch size mismatch")
        device = self._device_for(logits)
        if logits.device != device:
            logits = logits.to(device, non_blocking=True)
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        stream = torch.cuda.current_stream(device)
        if out is None:
            out = torch.empty(B, dtype=torch.int64, device=device)
        if B == 0:
            return out
        params = pack_params(all_sampling_params)
        temp = params[0]
        top_k = params[1].view(np.int32)
        sampled = temp != 0.0
        fast = sampled & (top_k > 0) & (top_k <= FAST_MAX_K) & (top_k.astype(np.int64) < self.vocab_total)
        general = np.nonzero(sampled & ~fast)[0].tolist()
        if cap is None:
            kmax = int(top_k[fast].max()) if fast.any() else 0
            cap = min(MAX_CAP, max(1, kmax + self.tie_slack))
        peer = self.transport == "peer"
        if peer:
            if self._exchange is None:
                self._exchange = PeerExchange(self.lib, self.group, self.world, self.rank, device)
            ex = self._exchange
            ex.ensure(B * (1 + cap), stream)
            ex.steps += 1
            par = ex.steps & 1
            rec_ptr = ex.record(self.rank, par)
        else:
            rec = torch.empty(B * (1 + cap), dtype=torch.int64, device=device)
            rec_ptr = rec.data_ptr()
        with self._lock:
            st = self._stage(device, B, all_generated_ids, all_sampling_params, uniforms, stream)
            if offset is None:
                offset = self.offset
                self.offset += 1
            ws = self._workspace.get(device.index)
            if ws is None:
                ws = self._workspace[device.index] = Workspace(device)
            ws_ptr, ws_bytes = ws.acquire(B, self.vocab_local, st.max_hist if st.hist_ids is not None else 0, stream)
            rc = self.lib.ns_vp_local(
                logits.data_ptr(), _DTYPES[logits.dtype], B, self.vocab_local, int(logits.stride(0)),
                self.vocab_offset, self.vocab_total,
                st.hist_ids, st.hist_offsets, st.max_hist,
                st.p32, st.p32 + 4 * B, st.p32 + 8 * B, st.p32 + 12 * B, st.p32 + 16 * B, st.p32 + 20 * B,
                cap, rec_ptr, ws_ptr, ws_bytes, stream.cuda_stream)
            ws.release(stream)
            if rc != _lib.NS_OK:
                raise RuntimeError(f"ns_vp_local failed: {_lib.status_string(rc)}")
            if peer:
                flags, _keep1 = _ptr_array([ex.flags(r) for r in range(self.world)])
                rc = self.lib.ns_vp_signal(flags, self.world, self.rank, ex.counter(), stream.cuda_stream)
                if rc != _lib.NS_OK:
                    raise RuntimeError(f"ns_vp_signal failed: {_lib.status_string(rc)}")
                recs, _keep2 = _ptr_array([ex.record(r, par) for r in range(self.world)])

                def merge():
                    return self.lib.ns_vp_merge_peers(
                        recs, self.world, ex.flags(self.rank), ex.counter(), B, cap, self.vocab_total,
                        st.p32, st.p32 + 4 * B, st.p32 + 8 * B, st.u_ptr, self.seed, offset,
                        out.data_ptr(), stream.cuda_stream)
                rc = merge()
                if rc == _lib.NS_OK and bool((out == _lib.NS_ERR_DEVICE_TIMEOUT).any()):
                    rc = self._recover_timeout(ex, stream, merge, out)
            else:
                gathered = gather_records(rec, self.group)
                rc = self.lib.ns_vp_merge(
                    gathered.data_ptr(), self.world, B, cap, self.vocab_total,
                    st.p32, st.p32 + 4 * B, st.p32 + 8 * B, st.u_ptr, self.seed, offset,
                    out.data_ptr(), stream.cuda_stream)
            st.keep_alive(stream)
            if rc != _lib.NS_OK:
                raise RuntimeError(f"ns_vp_merge failed: {_lib.status_string(rc)}")
        if general:
            idx = torch.tensor(general, dtype=torch.long, device=device)
            full = gather_full_rows(logits.index_select(0, idx), self.offsets, self.widths, self.vocab_total,
                                    self.group)
            hs = None if all_generated_ids is None else [all_generated_ids[b] for b in general]
            ps = [all_sampling_params[b] for b in general]
            us = None if uniforms is None else uniforms.reshape(-1)[idx.to(uniforms.device)]
            sub = B200Sampler.select_batch_tensor(self, full, hs, ps, uniforms=us)
            out.index_copy_(0, idx, sub)
        if retry and cap < MAX_CAP:
            # every rank merged the same bytes, so every rank takes the same branch
            if bool((out == _lib.NS_ERR_CANDIDATE_OVERFLOW).any()):
                return self._run(logits, all_generated_ids, all_sampling_params, uniforms, out, retry=False,
                                 cap=MAX_CAP, offset=offset)
        return out
