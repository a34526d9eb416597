"""Per-row sampling parameters.

``SamplingParams`` mirrors ``nano_inference.core.sampling.SamplingParams``
(``src/nano_inference/core/sampling.py:4-12``) field for field and default for
default, and adds two fields the reference lacks: ``presence_penalty`` and
``frequency_penalty`` (default 0.0, which reproduces the reference exactly).
The sampler accepts any object with these attribute names, so the reference's
own ``SamplingParams`` instances work unchanged (missing extension fields read
as 0.0).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np


@dataclass
class SamplingParams:
    max_new_tokens: int = 256
    temperature: float = 0.7      # 0 = greedy
    top_k: int = -1               # <= 0 or >= vocab: disabled
    top_p: float = 1.0            # outside (0, 1): disabled
    repetition_penalty: float = 1.0
    presence_penalty: float = 0.0   # extension
    frequency_penalty: float = 0.0  # extension


# Row-parameter block uploaded to the device in one copy: six fp32 / int32
# columns of length B, in this order.
PARAM_COLUMNS = ("temperature", "top_k", "top_p", "repetition_penalty",
                 "presence_penalty", "frequency_penalty")


def pack_params(all_params: Sequence) -> np.ndarray:
    """Pack per-row params into a [6, B] 32-bit block: fp32 temperature, int32
    top_k, fp32 top_p, fp32 repetition/presence/frequency penalties.

    Temperatures are rounded to fp32 as the reference's ``temperatures``
    tensor is (``sampler.py:60-64``); a NaN or infinite temperature is rejected
    here because the reference's draw would raise on it."""
    B = len(all_params)
    out = np.empty((6, B), dtype=np.float32)
    temps = np.fromiter((float(p.temperature) for p in all_params), dtype=np.float64, count=B)
    if not np.isfinite(temps).all():
        raise RuntimeError("probability tensor contains either `inf`, `nan` or element < 0 "
                           "(non-finite temperature)")
    out[0] = temps.astype(np.float32)
    ks = np.fromiter((int(p.top_k) for p in all_params), dtype=np.int64, count=B)
    out[1].view(np.int32)[:] = np.clip(ks, -1, 2**31 - 1).astype(np.int32)
    out[2] = np.fromiter((float(p.top_p) for p in all_params), dtype=np.float64, count=B)
    out[3] = np.fromiter((float(p.repetition_penalty) for p in all_params), dtype=np.float64, count=B)
    out[4] = np.fromiter((float(getattr(p, "presence_penalty", 0.0) or 0.0) for p in all_params),
                         dtype=np.float64, count=B)
    out[5] = np.fromiter((float(getattr(p, "frequency_penalty", 0.0) or 0.0) for p in all_params),
                         dtype=np.float64, count=B)
    return out
