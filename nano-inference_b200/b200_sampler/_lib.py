"""ctypes binding of the C ABI declared in ``include/ns_sampler.h``.

The library is loaded from the package directory (built in-tree by
``b200_sampler.build``).  There is no fallback: if it is missing, loading
raises ``ImportError`` naming the build command.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

NS_OK = 0
NS_IPC_HANDLE_BYTES = 64
NS_NOALLOC_SCRATCH_BYTES = 16 << 20     # include/ns_sampler.h
NS_ERR_INVALID_ARGUMENT = -1
NS_ERR_WORKSPACE_TOO_SMALL = -2
NS_ERR_UNSUPPORTED_DTYPE = -3
NS_ERR_CUDA = -4
NS_ERR_DEVICE_TIMEOUT = -5
NS_ERR_TOKEN_ID_OUT_OF_RANGE = -6
NS_ERR_INVALID_DISTRIBUTION = -7
NS_ERR_HISTORY_TOO_LONG = -8
NS_ERR_CANDIDATE_OVERFLOW = -9
NS_ERR_UNSUPPORTED = -10

NS_DTYPE_F32 = 0
NS_DTYPE_BF16 = 1
NS_DTYPE_F16 = 2

# name -> (restype, argtypes); mirrors include/ns_sampler.h
_c_i64 = ctypes.c_int64
_c_u64 = ctypes.c_uint64
_c_int = ctypes.c_int
_c_vp = ctypes.c_void_p
_c_sz = ctypes.c_size_t

PROTOTYPES = {
    "ns_status_string": (ctypes.c_char_p, [_c_int]),
    "ns_version": (_c_int, []),
    "ns_sampler_workspace_bytes": (_c_int, [_c_i64, _c_i64, _c_i64, ctypes.POINTER(_c_sz)]),
    "ns_sampler_smem_bytes": (_c_int, [_c_int, _c_i64, _c_i64, _c_i64, _c_int, ctypes.POINTER(_c_sz)]),
    "ns_sample": (_c_int, [
        _c_vp, _c_int, _c_i64, _c_i64, _c_i64,       # logits, dtype, batch, vocab, row_stride
        _c_vp, _c_vp, _c_i64,                        # hist_ids, hist_offsets, max_history
        _c_vp, _c_vp, _c_vp,                         # temperature, top_k, top_p
        _c_vp, _c_vp, _c_vp,                         # repetition, presence, frequency
        _c_vp, _c_u64, _c_u64,                       # uniforms, philox_seed, philox_offset
        _c_vp, _c_vp, _c_sz, _c_vp,                  # out_ids, workspace, workspace_bytes, stream
    ]),
    "ns_sample_noalloc": (_c_int, [
        _c_vp, _c_int, _c_i64, _c_i64, _c_i64,       # logits, dtype, batch, vocab, row_stride
        _c_vp, _c_vp, _c_i64,                        # hist_ids, hist_offsets, max_history
        _c_vp, _c_vp, _c_vp,                         # temperature, top_k, top_p
        _c_vp, _c_vp, _c_vp,                         # repetition, presence, frequency
        _c_vp, _c_u64, _c_u64,                       # uniforms, philox_seed, philox_offset
        _c_vp, _c_vp,                                # out_ids, stream
    ]),
    "ns_hist_append": (_c_int, [
        _c_vp, _c_vp, _c_i64, _c_vp,                 # hist_ids, hist_offsets, batch, new_ids
        _c_vp, _c_vp, _c_i64, _c_vp,                 # out_hist_ids, out_hist_offsets, out_capacity, stream
    ]),
    "ns_vp_record_int64s": (_c_int, [_c_i64, _c_int, ctypes.POINTER(_c_i64)]),
    "ns_vp_local": (_c_int, [
        _c_vp, _c_int, _c_i64, _c_i64, _c_i64,       # logits, dtype, batch, vocab_local, row_stride
        _c_i64, _c_i64,                              # vocab_offset, vocab_total
        _c_vp, _c_vp, _c_i64,                        # hist_ids, hist_offsets, max_history
        _c_vp, _c_vp, _c_vp,                         # temperature, top_k, top_p
        _c_vp, _c_vp, _c_vp,                         # repetition, presence, frequency
        _c_int, _c_vp, _c_vp, _c_sz, _c_vp,          # cap, record, workspace, workspace_bytes, stream
    ]),
    "ns_vp_merge": (_c_int, [
        _c_vp, _c_int, _c_i64, _c_int, _c_i64,       # gathered, n_ranks, batch, cap, vocab_total
        _c_vp, _c_vp, _c_vp,                         # temperature, top_k, top_p
        _c_vp, _c_u64, _c_u64,                       # uniforms, philox_seed, philox_offset
        _c_vp, _c_vp,                                # out_ids, stream
    ]),
    "ns_vp_signal": (_c_int, [_c_vp, _c_int, _c_int, _c_vp, _c_vp]),    # rank_flags[], n, me, epoch, stream
    "ns_vp_merge_peers": (_c_int, [
        _c_vp, _c_int, _c_vp, _c_vp,                 # rank_records[], n_ranks, my_flags, epoch
        _c_i64, _c_int, _c_i64,                      # batch, cap, vocab_total
        _c_vp, _c_vp, _c_vp,                         # temperature, top_k, top_p
        _c_vp, _c_u64, _c_u64,                       # uniforms, philox_seed, philox_offset
        _c_vp, _c_vp,                                # out_ids, stream
    ]),
    "ns_penalize_debug": (_c_int, [
        _c_vp, _c_int, _c_i64, _c_i64, _c_i64,       # logits, dtype, batch, vocab, row_stride
        _c_vp, _c_vp,                                # hist_ids, hist_offsets
        _c_vp, _c_vp, _c_vp,                         # repetition, presence, frequency penalties
        _c_vp, _c_i64, _c_vp, _c_vp,                 # out, out_stride, row_status, stream
    ]),
    "ns_vp_peer_alloc": (_c_int, [_c_sz, ctypes.POINTER(_c_vp)]),
    "ns_vp_peer_free": (_c_int, [_c_vp]),
    "ns_ipc_handle": (_c_int, [_c_vp, _c_vp]),
    "ns_ipc_open": (_c_int, [_c_vp, ctypes.POINTER(_c_vp)]),
    "ns_ipc_close": (_c_int, [_c_vp]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the in-tree CUDA library (once)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"B200 sampler CUDA library not found at {LIB_PATH}; build it with "
                "`python -m b200_sampler.build` (from nano-inference_b200/) or "
                "`python -c 'import __graft_entry__ as g; g.build()'` at the repo root")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def status_string(code: int) -> str:
    return load().ns_status_string(int(code)).decode()


def workspace_bytes(batch: int, vocab: int, max_history: int) -> int:
    """Device workspace (bytes) an ns_sample / ns_vp_local call of this size needs."""
    n = ctypes.c_size_t()
    rc = load().ns_sampler_workspace_bytes(int(batch), int(vocab), int(max_history), ctypes.byref(n))
    if rc != NS_OK:
        raise ValueError(f"ns_sampler_workspace_bytes: {status_string(rc)}")
    return int(n.value)
