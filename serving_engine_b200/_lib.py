"""ctypes binding of the C ABI in ``include/serving_engine_b200.h``.

The shared library is built in-tree by ``serving_engine_b200.build``. There is
no fallback: if the library is missing or fails to load, ``lib()`` raises, so a
GPU path can never silently run something else.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_size_t, c_uint32, c_void_p

from .build import LIB_PATH

SEB_F32, SEB_F16, SEB_BF16 = 0, 1, 2
SEB_OK, SEB_EINVAL, SEB_EUNSUPPORTED, SEB_ECUDA, SEB_EWORKSPACE = 0, 1, 2, 3, 4
ERRBIT_BLOCK_ID, ERRBIT_SLOT, ERRBIT_TIMEOUT, ERRBIT_KLEN, ERRBIT_META = 1, 2, 4, 8, 16
ERRBIT_NAMES = {
    ERRBIT_BLOCK_ID: "block id out of range",
    ERRBIT_SLOT: "slot out of range",
    ERRBIT_TIMEOUT: "bounded wait timed out",
    ERRBIT_KLEN: "k_len exceeds block table row",
    ERRBIT_META: "row/query index out of range",
}

# name -> (restype, argtypes); must match include/serving_engine_b200.h
_I32P = POINTER(c_int32)
_I64P = POINTER(c_int64)
SIGNATURES = {
    "seb_version": (c_char_p, []),
    "seb_status_string": (c_char_p, [c_int32]),
    "seb_last_error": (c_char_p, []),
    "seb_kv_append": (
        c_int32,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p,
         c_void_p, c_int64, c_int32, c_int32, c_int32, c_void_p, c_void_p],
    ),
    "seb_copy_blocks": (
        c_int32,
        [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p,
         c_void_p],
    ),
    "seb_paged_decode_workspace_size": (c_int64, [c_int32, c_int32, c_int32, c_int32, c_int64, c_int32]),
    "seb_paged_decode": (
        c_int32,
        [c_void_p, c_int64, c_int64,            # q, strides
         c_void_p, c_void_p, c_int64,           # k_cache, v_cache, num_blocks
         c_void_p, c_int64, c_int64,            # block_table, stride, max_blocks
         c_void_p, c_void_p, c_void_p,          # q_starts, k_lens, q_pos_offsets
         c_int32, c_int32,                      # num_rows, total_query
         c_void_p, c_void_p, c_int32,           # item_query, item_row, num_items
         c_int32, c_int32, c_int32, c_int32,    # hq, hkv, head_dim, dtype
         c_float, c_int32, c_int32,             # scale, is_causal, blocks_per_split
         c_void_p, c_int64, c_int64,            # out, strides
         c_void_p, c_int64,                     # lse, stride
         c_void_p, c_int64, c_void_p, c_void_p],  # workspace, bytes, err, stream
    ),
    "seb_paged_prefill": (
        c_int32,
        [c_void_p, c_int64, c_int64,            # q, strides
         c_void_p, c_void_p, c_int64,           # k_cache, v_cache, num_blocks
         c_void_p, c_int64, c_int64,            # block_table, stride, max_blocks
         c_void_p, c_void_p, c_void_p, c_void_p,  # q_starts, q_lens, k_lens, q_pos_offsets
         c_int32, c_int32,                      # num_rows, total_query
         c_void_p, c_int32, c_int32,            # rows, num_prefill_rows, max_q_len
         c_int32, c_int32, c_int32, c_int32,    # hq, hkv, head_dim, dtype
         c_float, c_int32,                      # scale, is_causal
         c_void_p, c_int64, c_int64,            # out, strides
         c_void_p, c_int64,                     # lse, stride
         c_void_p, c_void_p],                   # err, stream
    ),
    "seb_paged_attention_workspace_size": (c_int64, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int64]),
    "seb_paged_attention": (
        c_int32,
        [c_void_p, c_int64, c_int64,            # q, strides
         c_void_p, c_void_p, c_int64,           # k_cache, v_cache, num_blocks
         c_void_p, c_int64, c_int64,            # block_table, stride, max_blocks
         c_void_p, c_void_p, c_void_p, c_void_p,  # q_lens, k_lens, q_starts, q_pos_offsets
         c_int32, c_int32,                      # num_rows, total_query
         c_int32, c_int32, c_int32, c_int32,    # hq, hkv, head_dim, dtype
         c_float, c_int32,                      # scale, is_causal
         c_void_p, c_int64, c_int64,            # out, strides
         c_void_p, c_int64,                     # lse, stride
         c_void_p, c_int64, c_void_p, c_void_p],  # workspace, bytes, err, stream
    ),
    # seb_paged_decode without the workspace pair (built-in scratch)
    "seb_paged_decode_noalloc": (
        c_int32,
        [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int64,
         c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_int32,
         c_int32, c_int32, c_int32, c_int32, c_float, c_int32, c_int32,
         c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p],
    ),
    "seb_rope_kv_append": (
        c_int32,
        [c_void_p, c_int64, c_int64, c_int32, c_int32, c_int32,  # qkv, stride, n_tokens, hq, hkv, head_dim
         c_void_p, c_void_p, c_int64,                            # cos, sin, stride
         c_void_p, c_void_p, c_int64,                            # slot_mapping, q_out, stride
         c_void_p, c_void_p, c_int64, c_int32, c_void_p, c_void_p],  # k_cache, v_cache, num_blocks, dtype, err, stream
    ),
    "seb_add_rmsnorm": (
        c_int32,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int32, c_float, c_int32,
         c_void_p],
    ),
    "seb_swiglu": (c_int32, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int32, c_int32, c_void_p]),
    "seb_selftest_bounded_wait": (c_int32, [c_uint32, c_void_p, c_void_p]),
    "seb_peer_alloc": (c_int32, [c_size_t, POINTER(c_void_p)]),
    "seb_peer_free": (c_int32, [c_void_p]),
    "seb_peer_export": (c_int32, [c_void_p, c_void_p]),
    "seb_peer_import": (c_int32, [c_void_p, POINTER(c_void_p)]),
    "seb_peer_close": (c_int32, [c_void_p]),
    "seb_allreduce_add_rmsnorm": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p,  # partial, x, out, flags (host arrays of device pointers)
         c_void_p, c_int64, c_int32, c_float,     # weight, n_tokens, hidden, eps
         c_int32, c_int32, c_int32, c_int32,      # dtype, rank, world, all_ranks
         c_uint32, c_void_p, c_void_p],           # polls, err, stream
    ),
}
SEB_MAX_PEERS = 8
SEB_PEER_HANDLE_BYTES = 64
SEB_PEER_FLAG_BYTES = 1024
NOALLOC_SCRATCH_BYTES = 32 << 20  # SEB_NOALLOC_SCRATCH_BYTES

_LIB: ctypes.CDLL | None = None


class SebError(RuntimeError):
    """A C-ABI call returned a non-OK status."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn}: {message or 'error'} (status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the shared library once; raise if it is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = os.environ.get("SEB_LIBRARY", str(LIB_PATH))
    if not os.path.exists(path):
        raise ImportError(
            f"serving_engine_b200: CUDA library not built ({path} missing); "
            "run `python -m serving_engine_b200.build`")
    handle = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = handle
    return handle


def check(fn: str, status: int) -> None:
    if status == SEB_OK:
        return
    msg = lib().seb_last_error().decode(errors="replace")
    if status in (SEB_EINVAL, SEB_EWORKSPACE):
        raise ValueError(f"{fn}: {msg} (status {status})")
    raise SebError(fn, status, msg)


def decode_errbits(bits: int) -> list[str]:
    return [name for bit, name in ERRBIT_NAMES.items() if bits & bit]
