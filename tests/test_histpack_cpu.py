"""The C-level history packer (host side of ``B200Sampler.select_batch``):
the same int32 CSR ids as a per-row numpy conversion, and the same errors
for ids that cannot be token ids."""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "nano-inference_b200"))


@pytest.fixture(scope="module")
def pack():
    from b200_sampler import build
    build.build_histpack()
    from b200_sampler._histpack import pack
    return pack


def test_pack_matches_numpy(pack):
    rng = np.random.default_rng(0)
    rows = [list(map(int, rng.integers(-5, 2 ** 31 - 1, size=int(n)))) for n in rng.integers(0, 300, size=50)]
    rows[3] = []
    rows[7] = [2 ** 31 - 1, -2 ** 31, 0, 1 << 29, (1 << 30) + 7]   # compact and multi-digit ints
    rows[9] = (np.int64(5), np.int32(6), True)                       # any __index__ objects in any sequence
    total = sum(len(r) for r in rows)
    out = np.full(total + 4, -7, dtype=np.int32)
    assert pack(rows, out) == total
    ref = np.concatenate([np.asarray([int(v) for v in r], dtype=np.int64) for r in rows]).astype(np.int32)
    assert (out[:total] == ref).all() and (out[total:] == -7).all()


def test_pack_errors(pack):
    out = np.zeros(8, dtype=np.int32)
    with pytest.raises(OverflowError):
        pack([[1, 2 ** 31]], out)
    with pytest.raises(OverflowError):
        pack([[-(2 ** 31) - 1]], out)
    with pytest.raises(TypeError):
        pack([[1, 2.5]], out)
    with pytest.raises(TypeError):
        pack([[1, "3"]], out)
    with pytest.raises(ValueError):
        pack([[1] * 9], out)          # never writes past the buffer
    with pytest.raises(TypeError):
        pack(5, out)
