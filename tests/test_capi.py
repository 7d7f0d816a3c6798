"""The C-ABI library loads, exports every symbol the header declares, and its
host-side argument checks reject bad calls before touching the GPU."""
import ctypes
import re
from pathlib import Path

import pytest

from serving_engine_b200 import _lib
from serving_engine_b200.build import LIB_PATH, build

HEADER = Path(__file__).resolve().parent.parent / "include" / "serving_engine_b200.h"


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.lib()


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(seb_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("seb_kv_append", "seb_copy_blocks", "seb_paged_decode", "seb_paged_decode_workspace_size",
              "seb_last_error", "seb_version", "seb_status_string"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    assert LIB_PATH.exists()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_only_c_abi_symbols_are_exported(lib):
    """Every seb_* symbol the library exports is declared in the header."""
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line and "seb_" in line}
    assert exported <= set(declared_functions()), exported - set(declared_functions())


def test_version_and_status_strings(lib):
    assert b"sm_100a" in lib.seb_version()
    assert lib.seb_status_string(_lib.SEB_EINVAL) == b"invalid argument"
    assert lib.seb_status_string(_lib.SEB_EWORKSPACE) == b"workspace too small"


def test_kv_append_rejects_bad_dtype_without_gpu(lib):
    st = lib.seb_kv_append(1024, 64, 64, 1024, 64, 64, 4, 2048, 4096, 8192, 8, 1, 64, 99, None, None)
    assert st == _lib.SEB_EINVAL
    assert b"dtype" in lib.seb_last_error()


def test_kv_append_zero_tokens_is_noop(lib):
    assert lib.seb_kv_append(None, 0, 0, None, 0, 0, 0, None, None, None, 8, 1, 64, _lib.SEB_BF16, None, None) == 0


def test_kv_append_rejects_null(lib):
    st = lib.seb_kv_append(None, 64, 64, None, 64, 64, 4, None, None, None, 8, 1, 64, _lib.SEB_BF16, None, None)
    assert st == _lib.SEB_EINVAL and b"NULL" in lib.seb_last_error()


def test_copy_blocks_validation(lib):
    assert lib.seb_copy_blocks(None, 2, 0, 8, 4096, None, None, 0, None, None) == 0
    assert lib.seb_copy_blocks(None, 2, 0, 8, 4096, None, None, 3, None, None) == _lib.SEB_EINVAL


def _decode_args(**over):
    a = dict(q=4096, qs=4096, qh=128, kc=1 << 20, vc=1 << 21, nb=64, bt=8192, bts=8, mb=8, qst=9000, kl=9100,
             qp=9200, rows=2, tq=2, iq=None, ir=None, items=2, hq=32, hkv=8, d=128, dtype=_lib.SEB_BF16,
             scale=0.088, causal=1, bps=0, out=1 << 22, os=4096, oh=128, lse=1 << 23, ls=32, ws=None, wsb=0,
             err=None, stream=None)
    a.update(over)
    return list(a.values())


def test_paged_decode_validation(lib):
    assert lib.seb_paged_decode(*_decode_args(items=0)) == 0
    assert lib.seb_paged_decode(*_decode_args(hq=30)) == _lib.SEB_EINVAL
    assert b"multiple" in lib.seb_last_error()
    assert lib.seb_paged_decode(*_decode_args(hq=64, hkv=2)) == _lib.SEB_EINVAL  # group 32 > 16
    assert lib.seb_paged_decode(*_decode_args(kc=(1 << 20) + 8)) == _lib.SEB_EINVAL  # misaligned pool
    assert lib.seb_paged_decode(*_decode_args(bts=4)) == _lib.SEB_EINVAL  # stride < max_blocks
    assert lib.seb_paged_decode(*_decode_args(dtype=7)) == _lib.SEB_EINVAL
    # split-K needed (max_blocks 512) but no workspace
    assert lib.seb_paged_decode(*_decode_args(mb=512, bts=512)) == _lib.SEB_EWORKSPACE


def test_decode_workspace_size(lib):
    assert lib.seb_paged_decode_workspace_size(0, 32, 8, 128, 512, 0) == 0
    # one split per item -> no workspace
    assert lib.seb_paged_decode_workspace_size(64, 32, 8, 128, 8, 8) == 0
    n = lib.seb_paged_decode_workspace_size(64, 32, 8, 128, 512, 32)
    # partial O and (m, l) per split, then one int32 counter per (item, kv head)
    assert n == 64 * 32 * 16 * (128 + 2) * 4 + 64 * 8 * 4


def test_ctypes_signatures_match_header_arity():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, (_, args) in _lib.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\(([^;]*)\)\s*;", text)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), (name, len(params), len(args))


def _ar_args(world=2, hidden=512, dtype=None, ptr=1 << 20, weight=1 << 21, rank=0, all_ranks=0):
    """Arguments of seb_allreduce_add_rmsnorm with host pointer arrays of fake,
    16-byte aligned device addresses (validation never dereferences them)."""
    arr = lambda: (ctypes.c_void_p * max(world, 1))(*[ptr + 4096 * q for q in range(max(world, 1))])
    return (arr(), arr(), arr(), arr(), weight, 256, hidden, ctypes.c_float(1e-5),
            _lib.SEB_BF16 if dtype is None else dtype, rank, world, all_ranks, 0, None, None)


def test_allreduce_add_rmsnorm_validation(lib):
    assert lib.seb_allreduce_add_rmsnorm(*_ar_args(world=_lib.SEB_MAX_PEERS + 1)) == _lib.SEB_EINVAL
    assert b"world" in lib.seb_last_error()
    assert lib.seb_allreduce_add_rmsnorm(*_ar_args(world=0)) == _lib.SEB_EINVAL
    assert lib.seb_allreduce_add_rmsnorm(*_ar_args(hidden=500)) == _lib.SEB_EINVAL  # not a multiple of 8
    assert b"hidden" in lib.seb_last_error()
    assert lib.seb_allreduce_add_rmsnorm(*_ar_args(dtype=_lib.SEB_F32)) == _lib.SEB_EINVAL
    assert lib.seb_allreduce_add_rmsnorm(*_ar_args(rank=2)) == _lib.SEB_EINVAL  # rank outside the world
    assert lib.seb_allreduce_add_rmsnorm(*_ar_args(rank=1, all_ranks=1)) == _lib.SEB_EINVAL
    assert lib.seb_allreduce_add_rmsnorm(*_ar_args(ptr=(1 << 20) + 8)) == _lib.SEB_EINVAL  # misaligned buffers
    assert b"aligned" in lib.seb_last_error()
    assert lib.seb_allreduce_add_rmsnorm(*_ar_args(weight=0)) == _lib.SEB_EINVAL
    assert b"NULL" in lib.seb_last_error()


def test_peer_memory_calls_reject_null(lib):
    assert lib.seb_peer_alloc(0, None) == _lib.SEB_EINVAL
    assert lib.seb_peer_export(None, None) == _lib.SEB_EINVAL
    assert lib.seb_peer_import(None, None) == _lib.SEB_EINVAL


def test_paged_attention_workspace_size(lib):
    """The routed entry point's workspace: the routing region (two counts, decode
    items' tokens and rows, the prefill unit list bounded by the host-known
    sizes), rounded to 256 bytes, then the split-K decode workspace for
    max(rows, total_query) items."""
    assert lib.seb_paged_attention_workspace_size(0, 10, 32, 8, 128, 64) == 0
    assert lib.seb_paged_attention_workspace_size(5, 0, 32, 8, 128, 64) == 0
    assert lib.seb_paged_attention_workspace_size(5, 100, 30, 8, 128, 64) == 0  # heads not a multiple
    rows, tq, hq, hkv, d, mb = 7, 1000, 32, 8, 128, 200
    pair_queries = 2 * (128 // (hq // hkv))
    cap = hkv * (tq // pair_queries + min(rows, tq // 2))
    route = 16 + 8 * rows + 8 * cap
    route = -(-route // 256) * 256
    decode = lib.seb_paged_decode_workspace_size(max(rows, tq), hq, hkv, d, mb, 0)
    assert lib.seb_paged_attention_workspace_size(rows, tq, hq, hkv, d, mb) == route + decode


def test_paged_attention_validation(lib):
    """Rejected on the host before any launch: NULL metadata, a workspace smaller
    than the size function reports, an unaligned workspace."""
    assert lib.seb_paged_attention(None, 0, 0, None, None, 1, None, 4, 4, None, None, None, None, 0, 0, 32, 8, 128,
                                   _lib.SEB_BF16, 0.1, 1, None, 0, 0, None, 0, None, 0, None, None) == _lib.SEB_OK
    st = lib.seb_paged_attention(None, 0, 0, None, None, 1, None, 4, 4, None, None, None, None, 3, 9, 32, 8, 128,
                                 _lib.SEB_BF16, 0.1, 1, None, 0, 0, None, 0, None, 0, None, None)
    assert st == _lib.SEB_EINVAL and b"NULL metadata" in lib.seb_last_error()
    fake = ctypes.c_void_p(4096)  # never dereferenced: the call returns before any launch
    need = lib.seb_paged_attention_workspace_size(3, 9, 32, 8, 128, 4)
    st = lib.seb_paged_attention(fake, 0, 0, fake, fake, 1, fake, 4, 4, fake, fake, fake, fake, 3, 9, 32, 8, 128,
                                 _lib.SEB_BF16, 0.1, 1, fake, 0, 0, fake, 0, fake, need - 16, None, None)
    assert st == _lib.SEB_EWORKSPACE
    st = lib.seb_paged_attention(fake, 0, 0, fake, fake, 1, fake, 4, 4, fake, fake, fake, fake, 3, 9, 32, 8, 128,
                                 _lib.SEB_BF16, 0.1, 1, fake, 0, 0, fake, 0, ctypes.c_void_p(4096 + 16), need,
                                 None, None)
    assert st == _lib.SEB_EWORKSPACE and b"256-byte aligned" in lib.seb_last_error()
