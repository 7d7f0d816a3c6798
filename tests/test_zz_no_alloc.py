"""The allocation-free decode entry point, seb_paged_decode_noalloc.

Some callers cannot give the library a workspace: their device memory is
owned by another allocator (the engine sizes its KV pool to most of the free
memory at start-up), or they bind the C ABI from a language with no access to
the framework's allocator. For them the library keeps its split-K scratch in a
fixed device array of its own.

These tests call that entry point through the C ABI on two different calls in
a row (the second one finds the first one's leftovers in the shared scratch)
and check that
  * it returns exactly what the workspace-taking seb_paged_decode returns (the
    same kernel with the same split length and a fixed merge order, so O and
    LSE must be bitwise equal),
  * sampled rows agree with the CPU oracle within the decode tolerance
    (tests/tolerance.py), so a fault shared by both entry points is caught too,
  * the device's free memory does not change across its calls: it allocates
    nothing.
The file runs last so a failure here cannot hide others.
"""
import numpy as np
import pytest
import torch

from oracle.paged_attention import decode_rows
from serving_engine_b200 import _lib, workloads
from serving_engine_b200.build import build
from serving_engine_b200.ops import decode_workspace_bytes, dtype_code
from serving_engine_b200.paged_attention import metadata_from_lists
from tests.tolerance import LSE_TOL, check_out

pytestmark = pytest.mark.gpu
SAMPLED_ROWS = (0, 5, 11)


def _common_args(b, md, q, out, lse):
    return [q.data_ptr(), q.stride(0), q.stride(1), b.k_cache.data_ptr(), b.v_cache.data_ptr(), b.k_cache.shape[0],
            md["block_table"].data_ptr(), md["block_table"].stride(0), md["block_table"].shape[1],
            md["q_starts"].data_ptr(), md["k_lens"].data_ptr(), md["q_pos_offsets"].data_ptr(),
            len(b.q_lens), q.shape[0], None, md["item_row"].data_ptr(), q.shape[0],
            b.num_q_heads, b.num_kv_heads, b.head_dim, dtype_code(q), b.scale, 1, 0,
            out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0)]


class _Case:
    """Device inputs and preallocated outputs of one decode batch."""

    def __init__(self, b):
        dev = torch.device("cuda", 0)
        self.b = b
        self.md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, dev)
        self.q = b.q.to(dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        ws_bytes = decode_workspace_bytes(self.q.shape[0], b.num_q_heads, b.num_kv_heads, b.head_dim,
                                          self.md["block_table"].shape[1])
        # split-K is in play, so the scratch is used, and it fits the built-in array
        assert 0 < ws_bytes <= _lib.NOALLOC_SCRATCH_BYTES
        self.ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        self.o_ws, self.l_ws = torch.empty_like(self.q), torch.empty(self.q.shape[0], b.num_q_heads,
                                                                      dtype=torch.float32, device=dev)
        self.o_na, self.l_na = torch.empty_like(self.q), torch.empty_like(self.l_ws)
        self.stream = torch.cuda.current_stream(dev).cuda_stream

    def run_workspace(self, lib):
        st = lib.seb_paged_decode(*_common_args(self.b, self.md, self.q, self.o_ws, self.l_ws), self.ws.data_ptr(),
                                  self.ws.numel(), self.err.data_ptr(), self.stream)
        assert st == 0, lib.seb_last_error()

    def run_noalloc(self, lib):
        st = lib.seb_paged_decode_noalloc(*_common_args(self.b, self.md, self.q, self.o_na, self.l_na),
                                          self.err.data_ptr(), self.stream)
        assert st == 0, lib.seb_last_error()


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row():
    build()
    lib = _lib.lib()
    cases = [_Case(workloads.decode_batch(16, 1024, 4096, 32, 8, 128, torch.bfloat16, seed=71, fill="cuda")),
             _Case(workloads.decode_batch(24, 300, 3000, 16, 4, 128, torch.bfloat16, seed=72, fill="cuda"))]
    for c in cases:
        c.run_workspace(lib)
    # The first call on the device looks the scratch up (the module may load
    # then); from there on no call may change the device's free memory.
    cases[0].run_noalloc(lib)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for c in cases:  # the second call finds the first one's leftovers in the scratch
        c.run_noalloc(lib)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, f"free device memory changed by {free_before - free_after} bytes"
    for c in cases:
        assert int(c.err.item()) == 0
        assert torch.equal(c.o_na.view(torch.int16), c.o_ws.view(torch.int16)), "O differs from seb_paged_decode"
        assert torch.equal(c.l_na, c.l_ws), "LSE differs from seb_paged_decode"
        b = c.b
        ref = decode_rows(b.q, b.k_cache, b.v_cache, b.block_tables, b.k_lens, b.scale, SAMPLED_ROWS)
        for r in SAMPLED_ROWS:
            o_ref, lse_ref = ref[r]
            ok, msg = check_out(c.o_na[r].float().cpu().numpy(), o_ref, torch.bfloat16)
            assert ok, f"row {r}: {msg}"
            np.testing.assert_allclose(c.l_na[r].cpu().numpy(), lse_ref, atol=LSE_TOL["bf16"], rtol=0)


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
    msg = lib.seb_last_error()
    assert b"built-in scratch" in msg and b"capped at 64" in msg
