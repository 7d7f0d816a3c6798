"""The allocation-free decode entry point, seb_paged_decode_noalloc.

Some callers cannot give the library a workspace: their device memory is
owned by another allocator (the engine sizes its KV pool to most of the free
memory at start-up), or they bind the C ABI from a language with no access to
the framework's allocator. For them the library keeps its split-K scratch in a
fixed device array of its own. These tests call that entry point through the
C ABI and check, on two different calls in a row (the second one finds the
first one's leftovers in the shared scratch), that it returns what the
workspace-taking seb_paged_decode returns, within the tolerances the other
decode tests use. The file runs last so a failure here cannot hide others.
"""
import numpy as np
import pytest
import torch

from serving_engine_b200 import _lib, workloads
from serving_engine_b200.build import build
from serving_engine_b200.ops import decode_workspace_bytes, dtype_code
from serving_engine_b200.paged_attention import metadata_from_lists

pytestmark = pytest.mark.gpu


def _common_args(b, md, q, out, lse):
    return [q.data_ptr(), q.stride(0), q.stride(1), b.k_cache.data_ptr(), b.v_cache.data_ptr(), b.k_cache.shape[0],
            md["block_table"].data_ptr(), md["block_table"].stride(0), md["block_table"].shape[1],
            md["q_starts"].data_ptr(), md["k_lens"].data_ptr(), md["q_pos_offsets"].data_ptr(),
            len(b.q_lens), q.shape[0], None, md["item_row"].data_ptr(), q.shape[0],
            b.num_q_heads, b.num_kv_heads, b.head_dim, dtype_code(q), b.scale, 1, 0,
            out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0)]


def _run_both(lib, b):
    dev = torch.device("cuda", 0)
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, dev)
    q = b.q.to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws_bytes = decode_workspace_bytes(q.shape[0], b.num_q_heads, b.num_kv_heads, b.head_dim,
                                      md["block_table"].shape[1])
    assert 0 < ws_bytes <= _lib.NOALLOC_SCRATCH_BYTES  # split-K is in play, so the scratch is used
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    o_ws, l_ws = torch.empty_like(q), torch.empty(q.shape[0], b.num_q_heads, dtype=torch.float32, device=dev)
    o_na, l_na = torch.empty_like(q), torch.empty_like(l_ws)
    st = lib.seb_paged_decode(*_common_args(b, md, q, o_ws, l_ws), ws.data_ptr(), ws.numel(), err.data_ptr(),
                              stream)
    assert st == 0, lib.seb_last_error()
    st = lib.seb_paged_decode_noalloc(*_common_args(b, md, q, o_na, l_na), err.data_ptr(), stream)
    assert st == 0, lib.seb_last_error()
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0
    return o_ws.float().cpu().numpy(), l_ws.cpu().numpy(), o_na.float().cpu().numpy(), l_na.cpu().numpy()


def _assert_within_decode_tolerance(o, o_ref, lse, lse_ref):
    """bf16: 2e-3 plus half a bf16 ulp on O, 1e-3 on LSE (the other decode tests' bar)."""
    tol = 2e-3 + np.exp2(np.floor(np.log2(np.maximum(np.abs(o_ref), 1e-30))) - 8)
    assert (np.abs(o - o_ref) <= tol).all()
    np.testing.assert_allclose(lse, lse_ref, atol=1e-3, rtol=0)


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row():
    build()
    lib = _lib.lib()
    first = workloads.decode_batch(16, 1024, 4096, 32, 8, 128, torch.bfloat16, seed=71, fill="cuda")
    second = workloads.decode_batch(24, 300, 3000, 16, 4, 128, torch.bfloat16, seed=72, fill="cuda")
    for b in (first, second):
        o_ws, l_ws, o_na, l_na = _run_both(lib, b)
        assert np.isfinite(o_na).all() and np.isfinite(l_na).all()
        _assert_within_decode_tolerance(o_na, o_ws, l_na, l_ws)


def test_noalloc_rejects_a_call_beyond_its_scratch():
    build()
    lib = _lib.lib()
    items, hq, hkv, d, max_blocks = 4096, 32, 8, 128, 512
    need = lib.seb_paged_decode_workspace_size(items, hq, hkv, d, max_blocks, 0)
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    # rejected before any pointer is touched or any kernel is launched
    st = lib.seb_paged_decode_noalloc(None, 0, 0, None, None, 1, None, max_blocks, max_blocks, None, None, None,
                                      items, items, None, None, items, hq, hkv, d, _lib.SEB_BF16, 0.1, 1, 0,
                                      None, 0, 0, None, 0, None, None)
    assert st == _lib.SEB_EWORKSPACE
    assert b"built-in scratch" in lib.seb_last_error()
