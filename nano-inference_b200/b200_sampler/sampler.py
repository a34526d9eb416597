"""``B200Sampler``: drop-in replacement for nano-inference's ``Sampler``.

Keeps the reference call signature (``src/nano_inference/sampling/base.py:10-25``)::

    select(logits, generated_ids, sampling_params) -> int
    select_batch(logits, all_generated_ids, all_sampling_params) -> List[int]

and the engine's keyword call (``inferencer/torch_inferencer.py:254-258``), so
``inferencer.sampler = B200Sampler()`` is the whole integration.  Every row is
sampled on the GPU by the CUDA library behind ``include/ns_sampler.h``; the
host side only packs parameters and histories and reads back the ids.

Differences from the reference, all documented in the C header:

* the draw is an inverse-CDF draw from one uniform per row (caller supplied via
  ``uniforms=``, else a Philox4x32-10 stream keyed by ``seed``), not
  ``torch.multinomial``;
* ``presence_penalty`` / ``frequency_penalty`` are honoured when present on the
  params objects (default 0.0 reproduces the reference);
* the caller's logits are not modified (the reference penalises them in place,
  ``sampler.py:52``);
* a negative history id is an error (the reference's Python indexing wraps it).
"""
from __future__ import annotations

import array
import itertools
import threading
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _lib
from .params import pack_params
from .workspace import Workspace

try:  # C-level history packing (built with the library); array.array otherwise
    from ._histpack import pack as _pack_histories
except ImportError:  # pragma: no cover - a tree without the built packer
    _pack_histories = None

try:  # the reference's ABC when nano-inference is installed
    from nano_inference.sampling.base import SamplerBase  # type: ignore
except Exception:  # pragma: no cover - mirror of sampling/base.py:10-25
    from abc import ABC, abstractmethod

    class SamplerBase(ABC):
        @abstractmethod
        def select(self, logits: torch.Tensor, generated_ids: List[int], sampling_params) -> int: ...

        @abstractmethod
        def select_batch(self, logits: torch.Tensor, all_generated_ids: List[List[int]],
                         all_sampling_params) -> List[int]: ...


_DTYPES = {torch.float32: _lib.NS_DTYPE_F32, torch.bfloat16: _lib.NS_DTYPE_BF16,
           torch.float16: _lib.NS_DTYPE_F16}

_ROW_ERRORS = {
    _lib.NS_ERR_TOKEN_ID_OUT_OF_RANGE: IndexError,
}


def _align(n: int, a: int = 16) -> int:
    return (n + a - 1) // a * a


class _Staging:
    """Pinned host block + device block for one call's small inputs (params,
    history CSR, uniforms), uploaded with a single H2D copy."""

    def __init__(self, device: torch.device):
        self.device = device
        self.host = torch.empty(0, dtype=torch.uint8)
        self.dev = torch.empty(0, dtype=torch.uint8, device=device)
        self.event: Optional[torch.cuda.Event] = None

    def reserve(self, nbytes: int):
        if self.event is not None:
            self.event.synchronize()      # previous upload has left the host block
        if self.host.numel() < nbytes:
            cap = max(nbytes, 2 * self.host.numel(), 1 << 16)
            self.host = torch.empty(cap, dtype=torch.uint8, pin_memory=True)
            self.dev = torch.empty(cap, dtype=torch.uint8, device=self.device)
        return self.host.numpy()

    def upload(self, nbytes: int, stream: torch.cuda.Stream):
        with torch.cuda.stream(stream):
            self.dev[:nbytes].copy_(self.host[:nbytes], non_blocking=True)
            if self.event is None:
                self.event = torch.cuda.Event()
            self.event.record(stream)
        return self.dev.data_ptr()


class _Staged:
    """Device pointers of one call's staged inputs."""

    def __init__(self, params, p32, hist_ids, hist_offsets, max_hist, u_ptr, u_dev):
        self.params = params          # host copy of the [6, B] block (numpy)
        self.p32 = p32
        self.hist_ids = hist_ids
        self.hist_offsets = hist_offsets
        self.max_hist = max_hist
        self.u_ptr = u_ptr
        self.u_dev = u_dev

    def keep_alive(self, stream: torch.cuda.Stream):
        if self.u_dev is not None:
            self.u_dev.record_stream(stream)


class B200Sampler(SamplerBase):
    """GPU sampler with the reference ``SamplerBase`` interface.

    Args:
        device: CUDA device for host-side inputs (default: the logits' device,
            else the current device).
        seed: Philox key for the default uniform stream.  Each call advances
            the stream's offset by one.
    """

    def __init__(self, device=None, seed: Optional[int] = None):
        self.lib = _lib.load()
        if not torch.cuda.is_available():
            raise RuntimeError("B200Sampler needs a CUDA device (there is no CPU fallback)")
        self.device = torch.device(device) if device is not None else None
        if seed is None:
            seed = int(torch.initial_seed()) & 0xFFFFFFFFFFFFFFFF
        self.seed = int(seed) & 0xFFFFFFFFFFFFFFFF
        self.offset = 0
        self._staging = {}
        self._workspace = {}  # device index -> Workspace
        self._landing = {}   # device index -> (device buffer for host logits, event after its last reader)
        self._lock = threading.Lock()

    # ------------------------------------------------------------------ API
    def select(self, logits: torch.Tensor, generated_ids: List[int], sampling_params,
               *, uniforms: Optional[torch.Tensor] = None) -> int:
        """Single-row sampling (reference ``Sampler.select``, sampler.py:11-34)."""
        if logits.dim() != 1:
            raise ValueError("select expects a 1-D logits row")
        u = None if uniforms is None else torch.as_tensor(uniforms, dtype=torch.float32).reshape(1)
        return self.select_batch(logits.unsqueeze(0), [generated_ids], [sampling_params], uniforms=u)[0]

    def select_batch(self, logits: torch.Tensor, all_generated_ids: List[List[int]],
                     all_sampling_params, *, uniforms: Optional[torch.Tensor] = None) -> List[int]:
        """Batch sampling (reference ``Sampler.select_batch``, sampler.py:36-91)."""
        ids = self.select_batch_tensor(logits, all_generated_ids, all_sampling_params, uniforms=uniforms)
        out = ids.tolist()
        bad = [v for v in out if v < 0]
        if bad:
            code = int(bad[0])
            exc = _ROW_ERRORS.get(code, RuntimeError)
            raise exc(_lib.status_string(code))
        return out

    def select_batch_tensor(self, logits: torch.Tensor, all_generated_ids: Optional[Sequence[Sequence[int]]],
                            all_sampling_params, *, uniforms: Optional[torch.Tensor] = None,
                            out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Like ``select_batch`` but asynchronous: returns int64 ids on the
        device (a negative entry is the ns_status of a failed row)."""
        if logits.dim() != 2:
            raise ValueError("select_batch expects [batch, vocab] logits")
        B, V = int(logits.shape[0]), int(logits.shape[1])
        if all_generated_ids is not None and len(all_generated_ids) != B:
            raise AssertionError("batch size mismatch (histories)")
        if len(all_sampling_params) != B:
            raise AssertionError("batch size mismatch (params)")
        if logits.dtype not in _DTYPES:
            raise TypeError(f"unsupported logits dtype {logits.dtype}")
        device = self._device_for(logits)
        stream = torch.cuda.current_stream(device)
        if logits.device == device and logits.stride(1) != 1:
            logits = logits.contiguous()
        if out is None:
            out = torch.empty(B, dtype=torch.int64, device=device)
        if B == 0:
            return out

        with self._lock:
            landed = None
            if logits.device != device:
                logits, landed = self._land(logits, device, stream)
            st = self._stage(device, B, all_generated_ids, all_sampling_params, uniforms, stream)
            offset = self.offset
            self.offset += 1
            ws = self._workspace.get(device.index)
            if ws is None:
                ws = self._workspace[device.index] = Workspace(device)
            ws_ptr, ws_bytes = ws.acquire(B, V, st.max_hist if st.hist_ids is not None else 0, stream)
            rc = self.lib.ns_sample(
                logits.data_ptr(), _DTYPES[logits.dtype], B, V, int(logits.stride(0)),
                st.hist_ids, st.hist_offsets, st.max_hist,
                st.p32, st.p32 + 4 * B, st.p32 + 8 * B,
                st.p32 + 12 * B, st.p32 + 16 * B, st.p32 + 20 * B,
                st.u_ptr, self.seed, offset,
                out.data_ptr(), ws_ptr, ws_bytes, stream.cuda_stream)
            ws.release(stream)
            st.keep_alive(stream)
            if landed is not None:
                landed.record(stream)   # the next call's copy waits for this launch
        if rc != _lib.NS_OK:
            raise RuntimeError(f"ns_sample failed: {_lib.status_string(rc)}")
        return out

    def penalized_logits(self, logits: torch.Tensor, all_generated_ids: Optional[Sequence[Sequence[int]]],
                         all_sampling_params) -> torch.Tensor:
        """Debug readback: fp32 [B, V] logits after the history penalties
        (repetition, frequency, presence; no temperature), bit for bit the
        values the sampling kernels use (``ns_penalize_debug``).  The
        reference applies the repetition step in place (sampler.py:52-57,
        93-108).  A history id outside [0, V) raises IndexError."""
        if logits.dim() != 2 or logits.dtype not in _DTYPES:
            raise ValueError("expected [batch, vocab] fp32 / bf16 / fp16 logits")
        B, V = int(logits.shape[0]), int(logits.shape[1])
        device = self._device_for(logits)
        stream = torch.cuda.current_stream(device)
        if logits.device != device or logits.stride(1) != 1:
            logits = logits.to(device).contiguous()
        out = torch.empty(B, V, dtype=torch.float32, device=device)
        status = torch.empty(B, dtype=torch.int32, device=device)
        if B == 0:
            return out
        with self._lock:
            st = self._stage(device, B, all_generated_ids, all_sampling_params, None, stream)
            rc = self.lib.ns_penalize_debug(
                logits.data_ptr(), _DTYPES[logits.dtype], B, V, int(logits.stride(0)),
                st.hist_ids, st.hist_offsets, st.p32 + 12 * B, st.p32 + 16 * B, st.p32 + 20 * B,
                out.data_ptr(), V, status.data_ptr(), stream.cuda_stream)
            st.keep_alive(stream)
        if rc != _lib.NS_OK:
            raise RuntimeError(f"ns_penalize_debug failed: {_lib.status_string(rc)}")
        bad = [int(v) for v in status.tolist() if v != _lib.NS_OK]
        if bad:
            raise _ROW_ERRORS.get(bad[0], RuntimeError)(_lib.status_string(bad[0]))
        return out

    def _stage(self, device: torch.device, B: int, all_generated_ids, all_sampling_params,
               uniforms: Optional[torch.Tensor], stream: torch.cuda.Stream) -> "_Staged":
        """Pack params [6, B], the history CSR (only when a row has a
        non-neutral penalty) and host uniforms into the pinned block, upload it
        with one copy, and return the device pointers.  Call under the lock."""
        params = pack_params(all_sampling_params)                       # [6, B] 32-bit
        use_hist = all_generated_ids is not None and bool(
            (params[3] != 1.0).any() or (params[4] != 0.0).any() or (params[5] != 0.0).any())
        if use_hist:
            lens = np.fromiter((len(h) for h in all_generated_ids), dtype=np.int64, count=B)
            total = int(lens.sum())
            max_hist = int(lens.max()) if B else 0
        else:
            total, max_hist = 0, 0
        host_u = uniforms is not None and uniforms.device.type == "cpu"

        off_params = 0
        off_offsets = _align(6 * B * 4)
        off_ids = _align(off_offsets + (B + 1) * 8)
        off_u = _align(off_ids + total * 4)
        nbytes = _align(off_u + (B * 4 if host_u else 0))

        stg = self._staging_for(device)
        h = stg.reserve(nbytes)
        h[off_params:off_params + 6 * B * 4] = params.reshape(-1).view(np.uint8)
        if use_hist and total:
            offs = h[off_offsets:off_offsets + (B + 1) * 8].view(np.int64)
            offs[0] = 0
            np.cumsum(lens, out=offs[1:])
            ids32 = h[off_ids:off_ids + total * 4].view(np.int32)
            try:  # ids beyond int32 cannot be token ids
                if _pack_histories is not None:
                    _pack_histories(all_generated_ids, ids32)
                else:
                    pos = 0
                    for row in all_generated_ids:
                        n = len(row)
                        if n:
                            ids32[pos:pos + n] = np.frombuffer(array.array("i", row), dtype=np.int32)
                            pos += n
            except OverflowError:
                raise IndexError(_lib.status_string(_lib.NS_ERR_TOKEN_ID_OUT_OF_RANGE)) from None
        if host_u:
            hu = uniforms.detach().to(torch.float32).reshape(-1).numpy()
            if hu.size != B:
                raise ValueError("uniforms must have one value per row")
            h[off_u:off_u + B * 4].view(np.float32)[:] = hu
        base = stg.upload(nbytes, stream)

        ud = None
        if uniforms is None:
            u_ptr = None
        elif host_u:
            u_ptr = base + off_u
        else:
            ud = uniforms.to(device=device, dtype=torch.float32).reshape(-1).contiguous()
            if ud.numel() != B:
                raise ValueError("uniforms must have one value per row")
            u_ptr = ud.data_ptr()
        has = use_hist and total > 0
        return _Staged(params=params, p32=base + off_params,
                       hist_ids=(base + off_ids) if has else None,
                       hist_offsets=(base + off_offsets) if has else None,
                       max_hist=max_hist, u_ptr=u_ptr, u_dev=ud)

    # -------------------------------------------------------------- helpers
    def _land(self, logits: torch.Tensor, device: torch.device, stream: torch.cuda.Stream):
        """Copy host (or other-device) logits into a per-device buffer that is
        kept between calls: a fresh allocation per call roughly quarters the
        pinned host-to-device rate.  Returns the device view and the event to
        record after the launch that reads it.  Call under the lock."""
        buf, ev = self._landing.get(device.index, (None, None))
        need = logits.numel()
        if buf is None or buf.numel() < need or buf.dtype != logits.dtype:
            if ev is not None:
                ev.synchronize()
            buf = torch.empty(max(need, 1), dtype=logits.dtype, device=device)
            ev = torch.cuda.Event()
            self._landing[device.index] = (buf, ev)
        else:
            stream.wait_event(ev)   # the previous reader of the buffer is done
        dst = buf[:need].view(logits.shape)
        with torch.cuda.stream(stream):
            dst.copy_(logits, non_blocking=True)
        return dst, ev

    def _device_for(self, logits: torch.Tensor) -> torch.device:
        if logits.is_cuda:
            return logits.device
        if self.device is not None:
            return self.device
        return torch.device("cuda", torch.cuda.current_device())

    def _staging_for(self, device: torch.device) -> _Staging:
        key = device.index
        if key not in self._staging:
            self._staging[key] = _Staging(device)
        return self._staging[key]


class DeviceBatch:
    """Device-resident per-row inputs (params, history CSR, optional uniforms)
    for repeated launches on logits that change every step -- the shape of a
    decode loop whose histories live on the GPU.  ``launch`` is one
    ``ns_sample`` call with no host work, so it can be captured in a CUDA
    graph (after a first launch outside the capture has allocated the
    workspace).  The batch owns its workspace: launches of one DeviceBatch
    must not overlap on the device."""

    def __init__(self, histories: Optional[Sequence[Sequence[int]]], params, device,
                 uniforms: Optional[torch.Tensor] = None, seed: int = 0,
                 history: Optional["DeviceHistory"] = None):
        self.lib = _lib.load()
        self.device = torch.device(device)
        self.batch = len(params)
        self.params = torch.from_numpy(pack_params(params)).to(self.device)      # [6, B]
        self.seed = seed
        self.history = history   # a DeviceHistory replaces `histories` when given
        B = self.batch
        if history is not None:
            if histories is not None:
                raise ValueError("pass histories or a DeviceHistory, not both")
            if history.batch != B:
                raise AssertionError("batch size mismatch (history)")
        if histories is not None and any(len(h) for h in histories):
            lens = np.array([len(h) for h in histories], dtype=np.int64)
            offs = np.zeros(B + 1, dtype=np.int64)
            np.cumsum(lens, out=offs[1:])
            flat = np.fromiter(itertools.chain.from_iterable(histories), dtype=np.int64, count=int(lens.sum()))
            self.hist_ids = torch.from_numpy(flat.astype(np.int32)).to(self.device)
            self.hist_offsets = torch.from_numpy(offs).to(self.device)
            self.max_history = int(lens.max())
        else:
            self.hist_ids = self.hist_offsets = None
            self.max_history = 0
        self.uniforms = None if uniforms is None else uniforms.to(self.device, torch.float32).contiguous()
        self.workspace = Workspace(self.device)

    def nbytes(self) -> int:
        """Bytes of the per-row inputs (params, history CSR, uniforms)."""
        n = self.params.numel() * 4
        if self.hist_ids is not None:
            n += self.hist_ids.numel() * 4 + self.hist_offsets.numel() * 8
        if self.uniforms is not None:
            n += self.uniforms.numel() * 4
        return n

    def launch(self, logits: torch.Tensor, out: torch.Tensor, stream: Optional[torch.cuda.Stream] = None,
               offset: int = 0) -> int:
        B, V = logits.shape
        assert B == self.batch and logits.stride(1) == 1 and out.numel() >= B
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        p = self.params.data_ptr()
        if self.history is not None:
            h = self.history
            hist_ids, hist_offsets, max_h = h.ids.data_ptr(), h.offsets.data_ptr(), h.max_history
        elif self.hist_ids is not None:
            hist_ids, hist_offsets, max_h = self.hist_ids.data_ptr(), self.hist_offsets.data_ptr(), self.max_history
        else:
            hist_ids, hist_offsets, max_h = None, None, 0
        ws_ptr, ws_bytes = self.workspace.acquire(B, V, max_h)
        return self.lib.ns_sample(
            logits.data_ptr(), _DTYPES[logits.dtype], B, V, int(logits.stride(0)),
            hist_ids, hist_offsets, max_h, p, p + 4 * B, p + 8 * B, p + 12 * B, p + 16 * B, p + 20 * B,
            None if self.uniforms is None else self.uniforms.data_ptr(), self.seed, offset,
            out.data_ptr(), ws_ptr, ws_bytes, s.cuda_stream)


class DeviceHistory:
    """Token histories (prompt + outputs per row) kept on the device for a
    decode loop.

    The reference rebuilds every row's history on the host each step --
    ``prompt_token_ids + output_token_ids`` (engine/context_builder.py:208-213),
    the sampled id appended to the outputs (driver/output_processor.py:46) --
    and the sampler re-uploads it.  Here the history is a CSR (int32 ids,
    int64 offsets) in device memory; ``append(ids)`` adds each row's sampled
    id with one ``ns_hist_append`` launch on the stream: no host work, no
    synchronisation, so a decode step can be captured in a CUDA graph once the
    buffers are large enough.  Two buffers alternate (the kernel reads one and
    writes the other); ``reserve_steps`` appends fit before a buffer grows, and
    growing allocates (keep it outside graph capture).  A failed row's
    negative status is appended as -1, which the next sampling step reports
    as NS_ERR_TOKEN_ID_OUT_OF_RANGE.
    """

    def __init__(self, histories: Sequence[Sequence[int]], device, reserve_steps: int = 256):
        self.lib = _lib.load()
        self.device = torch.device(device)
        B = len(histories)
        self.batch = B
        lens = np.fromiter((len(h) for h in histories), dtype=np.int64, count=B)
        offs = np.zeros(B + 1, dtype=np.int64)
        np.cumsum(lens, out=offs[1:])
        self.total = int(offs[-1])
        self.max_history = int(lens.max()) if B else 0
        flat = np.fromiter(itertools.chain.from_iterable(histories), dtype=np.int64, count=self.total)
        if flat.size and (flat.min() < -(2 ** 31) or flat.max() >= 2 ** 31):
            raise IndexError(_lib.status_string(_lib.NS_ERR_TOKEN_ID_OUT_OF_RANGE))
        cap = self.total + B * max(int(reserve_steps), 1)
        self._ids = [torch.empty(max(cap, 1), dtype=torch.int32, device=self.device) for _ in range(2)]
        self._offs = [torch.empty(B + 1, dtype=torch.int64, device=self.device) for _ in range(2)]
        if self.total:
            self._ids[0][:self.total].copy_(torch.from_numpy(flat.astype(np.int32)))
        self._offs[0].copy_(torch.from_numpy(offs))
        self.cur = 0

    @property
    def ids(self) -> torch.Tensor:
        """int32 ids of the current CSR (the first ``total`` are valid)."""
        return self._ids[self.cur]

    @property
    def offsets(self) -> torch.Tensor:
        """int64 [batch + 1] row offsets of the current CSR."""
        return self._offs[self.cur]

    def append(self, new_ids: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Append new_ids[b] (int64 [batch] on the device, e.g. the sampler's
        output) to row b, asynchronously on `stream`."""
        B = self.batch
        if new_ids.dtype != torch.int64 or new_ids.numel() < B or not new_ids.is_cuda:
            raise ValueError("new_ids must be an int64 device tensor with one id per row")
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        nxt = 1 - self.cur
        need = self.total + B
        if self._ids[nxt].numel() < need:
            with torch.cuda.stream(s):
                self._ids[nxt] = torch.empty(max(need, 2 * self._ids[nxt].numel()), dtype=torch.int32,
                                             device=self.device)
        rc = self.lib.ns_hist_append(self._ids[self.cur].data_ptr(), self._offs[self.cur].data_ptr(), B,
                                     new_ids.data_ptr(), self._ids[nxt].data_ptr(), self._offs[nxt].data_ptr(),
                                     self._ids[nxt].numel(), s.cuda_stream)
        if rc != _lib.NS_OK:
            raise RuntimeError(f"ns_hist_append failed: {_lib.status_string(rc)}")
        self.cur = nxt
        self.total = need
        self.max_history += 1

    def to_lists(self) -> List[List[int]]:
        """The histories as Python lists (synchronises; for checking)."""
        ids = self.ids[:self.total].cpu().tolist()
        offs = self.offsets.cpu().tolist()
        return [ids[offs[b]:offs[b + 1]] for b in range(self.batch)]
