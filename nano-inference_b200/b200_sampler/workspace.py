"""Device workspace of the sampling calls (``ns_sampler_workspace_bytes``).

A call whose blocks meet more distinct history ids than shared memory keeps
(histories longer than 1024 ids) puts those blocks' rank arrays in a
caller-allocated device buffer.  ``Workspace`` keeps one buffer per device
between calls, grows it when a larger call needs more, and orders its users:
a call on another stream first waits for the previous call that used it.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib

_ALIGN = 256


class Workspace:
    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self.buf: Optional[torch.Tensor] = None
        self.event: Optional[torch.cuda.Event] = None

    def acquire(self, batch: int, vocab: int, max_history: int,
                stream: Optional[torch.cuda.Stream] = None) -> Tuple[int, int]:
        """(pointer, bytes) of a buffer large enough for the call; `stream`
        (when given) waits for the buffer's previous user."""
        need = max(_lib.workspace_bytes(batch, vocab, max_history), _ALIGN)
        if self.buf is None or self.buf.numel() - _ALIGN < need:
            if self.event is not None:
                self.event.synchronize()
            self.buf = torch.empty(need + _ALIGN, dtype=torch.uint8, device=self.device)
            self.event = None
        elif self.event is not None and stream is not None:
            stream.wait_event(self.event)
        base = self.buf.data_ptr()
        ptr = (base + _ALIGN - 1) // _ALIGN * _ALIGN
        return ptr, self.buf.numel() - (ptr - base)

    def release(self, stream: torch.cuda.Stream) -> None:
        """Record that the call just launched on `stream` uses the buffer."""
        if self.event is None:
            self.event = torch.cuda.Event()
        self.event.record(stream)
