"""C-ABI checks that need no GPU: the library loads, exports every function
declared in include/*.h, and rejects bad arguments before touching CUDA."""
import ctypes
import glob
import os
import re

import pytest
import torch

from b200_sampler import _lib
from b200_sampler.build import INCLUDE

pytestmark = pytest.mark.skipif(not os.path.exists(_lib.LIB_PATH), reason="library not built")


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(INCLUDE, "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(ns_[a-z_0-9]+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert {"ns_sample", "ns_sampler_workspace_bytes", "ns_status_string", "ns_version"} <= names
    for n in names:
        assert hasattr(lib, n), n
    assert set(_lib.PROTOTYPES) >= names


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.ns_version() >= 100
    for code in range(-10, 1):
        assert lib.ns_status_string(code)
    assert _lib.status_string(_lib.NS_ERR_INVALID_DISTRIBUTION).startswith("probability tensor")


def test_workspace_query():
    lib = _lib.load()
    sz = ctypes.c_size_t(123)
    assert lib.ns_sampler_workspace_bytes(256, 151936, 1024, ctypes.byref(sz)) == 0
    assert sz.value == 0                     # 1024 distinct ids fit a block's shared memory
    # longer histories: 12 B per block per min(max_history, columns of a
    # block).  Without a device the widest clusters the vocabulary allows are
    # assumed: 8 blocks of 19456 columns per row at vocab 151936.
    assert lib.ns_sampler_workspace_bytes(256, 151936, 32768, ctypes.byref(sz)) == 0
    if not torch.cuda.is_available():
        assert sz.value == 256 * 8 * 12 * 19456
    assert sz.value >= 256 * 12 * 32768      # at least one block per row
    assert _lib.workspace_bytes(256, 151936, 1025) > 0
    assert lib.ns_sampler_workspace_bytes(-1, 10, 0, ctypes.byref(sz)) == _lib.NS_ERR_INVALID_ARGUMENT
    assert lib.ns_sampler_workspace_bytes(1, 1 << 25, 0, ctypes.byref(sz)) == _lib.NS_ERR_INVALID_ARGUMENT


def _call(**kw):
    lib = _lib.load()
    a = dict(logits=1, dtype=0, batch=1, vocab=10, row_stride=10, hist_ids=None, hist_offsets=None,
             max_history=0, temperature=1, top_k=1, top_p=1, rep=None, pres=None, freq=None,
             uniforms=None, seed=0, offset=0, out=1, ws=None, ws_bytes=0, stream=None)
    a.update(kw)
    return lib.ns_sample(*a.values())


def test_argument_validation_without_gpu():
    assert _call(dtype=7) == _lib.NS_ERR_UNSUPPORTED_DTYPE
    assert _call(vocab=0) == _lib.NS_ERR_INVALID_ARGUMENT
    assert _call(row_stride=5) == _lib.NS_ERR_INVALID_ARGUMENT
    assert _call(batch=-1) == _lib.NS_ERR_INVALID_ARGUMENT
    assert _call(hist_ids=1) == _lib.NS_ERR_INVALID_ARGUMENT        # ids without offsets
    assert _call(logits=None) == _lib.NS_ERR_INVALID_ARGUMENT
    assert _call(out=None) == _lib.NS_ERR_INVALID_ARGUMENT
    assert _call(batch=0, logits=None) == _lib.NS_OK                # empty batch: nothing to do


def test_package_has_no_oracle_dependency():
    pkg = os.path.dirname(_lib.__file__)
    for f in glob.glob(os.path.join(pkg, "*.py")):
        src = open(f).read()
        assert not re.search(r"^\s*(from\s+oracle|import\s+oracle)", src, flags=re.M), f


def test_hist_append_argument_validation_without_gpu():
    lib = _lib.load()
    f = lib.ns_hist_append
    assert f(None, None, -1, 1, 1, 1, 8, None) == _lib.NS_ERR_INVALID_ARGUMENT
    assert f(1, None, 2, 1, 1, 1, 8, None) == _lib.NS_ERR_INVALID_ARGUMENT      # ids without offsets
    assert f(None, None, 2, None, 1, 1, 8, None) == _lib.NS_ERR_INVALID_ARGUMENT  # no new ids
    assert f(None, None, 4, 1, 1, 1, 3, None) == _lib.NS_ERR_INVALID_ARGUMENT     # capacity below batch
    assert f(None, None, 0, None, None, None, 0, None) == _lib.NS_OK              # empty batch


def test_shared_memory_does_not_grow_with_the_history():
    """Two blocks per SM at any history length: the per-block shared memory
    of the headline shape (vocab 151936, batch 256, a 148-SM B200) is the same
    from 1024 to 32768 history ids and leaves room for a second block
    (228 KB per SM, 1 KB of it reserved per block)."""
    lib = _lib.load()
    sz = ctypes.c_size_t()
    sizes = {}
    for h in (1024, 2048, 11000, 12000, 32768):
        assert lib.ns_sampler_smem_bytes(_lib.NS_DTYPE_F32, 256, 151936, h, 148, ctypes.byref(sz)) == _lib.NS_OK
        sizes[h] = sz.value
    assert len(set(sizes.values())) == 1, sizes
    assert 2 * (sizes[1024] + 1024) <= 228 * 1024, sizes
    assert lib.ns_sampler_smem_bytes(_lib.NS_DTYPE_F32, 256, 151936, 0, 148, ctypes.byref(sz)) == _lib.NS_OK
    assert sz.value <= sizes[1024]                    # no history: no bitmap or rank arrays
    assert lib.ns_sampler_smem_bytes(7, 256, 151936, 0, 148, ctypes.byref(sz)) == _lib.NS_ERR_UNSUPPORTED_DTYPE
    assert lib.ns_sampler_smem_bytes(0, 0, 151936, 0, 148, ctypes.byref(sz)) == _lib.NS_ERR_INVALID_ARGUMENT
