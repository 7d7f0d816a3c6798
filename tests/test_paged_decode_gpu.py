"""Paged attention on the GPU (split-K decode kernel, through the C ABI) against
the CPU oracle and the reference's golden outputs.

Tolerances (tests/tolerance.py): fp32 outputs within max-abs 1e-5 of the
fp32/fp64 reference; bf16/fp16 outputs within max-abs 2e-3 of an fp32 reference
computed from the same 16-bit values wherever half an ulp of the stored type is
<= 1e-3 (bf16: |O| < 0.5), and 2e-3 plus half an ulp of the reference value
above that (the output's own final rounding). LSE is fp32 in every dtype: 1e-5
(fp32) / 1e-3 (16-bit inputs).
"""
import math

import numpy as np
import pytest
import torch

from oracle.paged_attention import decode_rows, paged_attention
from serving_engine_b200 import check_device_errors, paged_decode, paged_flash_attention, workloads
from serving_engine_b200.paged_attention import metadata_from_lists
from tests.golden.cases import attention_batches, noncausal_batch
from tests.tolerance import check_out
from tests.tolerance import out_tol as _out_tol

pytestmark = pytest.mark.gpu
DEV = "cuda"
LSE_TOL = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 1e-3}


def run_b200(b, is_causal=True, **kw):
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, DEV)
    q, kc, vc = b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV)
    if kw:
        o, lse = paged_decode(q, kc, vc, md["block_table"], md["q_starts"], md["k_lens"], md["q_pos_offsets"],
                              b.num_q_heads, b.num_kv_heads, b.scale, is_causal, item_row=md["item_row"], **kw)
    else:
        o, lse = paged_flash_attention(q, kc, vc, md, b.num_q_heads, b.num_kv_heads, b.scale, is_causal)
    torch.cuda.synchronize()
    check_device_errors()
    return o.float().cpu().numpy(), lse.cpu().numpy()


def run_oracle(b, is_causal=True):
    md = b.metadata("cpu")
    return paged_attention(b.q, b.k_cache, b.v_cache, md["block_table"], md["q_starts"], md["q_lens"],
                           md["k_lens"], md["q_pos_offsets"], b.scale, is_causal)


def out_tol(o_ref, dtype):
    """Plain 2e-3 (16-bit) / 1e-5 (fp32) where half an ulp of the stored type is
    <= 1e-3, else 2e-3 plus half an ulp of the reference value."""
    return _out_tol(o_ref, dtype)


def assert_out_close(o, o_ref, dtype):
    ok, msg = check_out(o, o_ref, dtype)
    assert ok, msg


def assert_close(o, lse, o_ref, lse_ref, dtype):
    assert_out_close(o, o_ref, dtype)
    np.testing.assert_allclose(lse, lse_ref, atol=LSE_TOL[dtype], rtol=0)


# ------------------------------------------------------------- golden vectors
@pytest.mark.parametrize("name", ["cfg1_fp32", "mixed_fp32"])
def test_matches_reference_triton_golden(name, golden_arrays):
    b, _ = attention_batches()[name]
    o, lse = run_b200(b)
    assert_close(o, lse, golden_arrays[f"{name}__triton_o"], golden_arrays[f"{name}__triton_lse"], torch.float32)
    np.testing.assert_allclose(o, golden_arrays[f"{name}__eager"], atol=1e-5, rtol=0)


def test_matches_reference_eager_bf16_golden(golden_arrays):
    b, _ = attention_batches()["gqa_bf16"]
    o, _ = run_b200(b)
    assert_out_close(o, golden_arrays["gqa_bf16__eager_fp32"], torch.bfloat16)


def test_noncausal_matches_reference_triton_golden(golden_arrays):
    o, lse = run_b200(noncausal_batch(), is_causal=False)
    assert_close(o, lse, golden_arrays["noncausal_fp32__triton_o"], golden_arrays["noncausal_fp32__triton_lse"],
                 torch.float32)


# ----------------------------------------------------------------- configs
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_config1_fp32(seed):
    b = workloads.config1(seed)
    o, lse = run_b200(b)
    o_ref, lse_ref = run_oracle(b)
    assert_close(o, lse, o_ref, lse_ref, torch.float32)


def test_config2_full_size_sampled_rows():
    """Full config-2 batch (64 seqs, k_len U[1024, 8192], 32/8 heads, D=128, bf16):
    every output finite; 8 sampled rows within 2e-3 of the fp64 oracle."""
    b = workloads.config2(seed=0, fill="cuda")
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, DEV)
    q = b.q.to(DEV)
    o, lse = paged_flash_attention(q, b.k_cache, b.v_cache, md, 32, 8, b.scale)
    torch.cuda.synchronize()
    check_device_errors()
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    rows = [0, 7, 13, 21, 34, 42, 55, 63]
    ref = decode_rows(b.q, b.k_cache, b.v_cache, b.block_tables, b.k_lens, b.scale, rows)
    for r in rows:
        o_ref, lse_ref = ref[r]
        assert_out_close(o[r].float().cpu().numpy(), o_ref, torch.bfloat16)
        np.testing.assert_allclose(lse[r].cpu().numpy(), lse_ref, atol=1e-3, rtol=0)


# ------------------------------------------------------------ shape coverage
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("hq,hkv", [(8, 8), (8, 4), (32, 8), (16, 2), (32, 2)])
@pytest.mark.parametrize("d", [64, 128, 256])
def test_shapes_vs_oracle(dtype, hq, hkv, d):
    b = workloads.decode_batch(5, 1, 300, hq, hkv, d, dtype, seed=hq * 7 + hkv + d, num_blocks=128)
    o, lse = run_b200(b)
    o_ref, lse_ref = run_oracle(b)
    assert_close(o, lse, o_ref, lse_ref, dtype)


@pytest.mark.parametrize("bps", [1, 3, 8, 32, 33, 40, 64, 100])
def test_split_sizes_agree(bps):
    """Every split size (1 block .. 64 blocks per split, the cap a larger request is
    held to; hence 1 .. many splits and the in-kernel merge of the splits; past 32
    blocks each lane holds a second block id) gives the oracle's answer."""
    b = workloads.decode_batch(6, 1, 1200, 32, 8, 128, torch.bfloat16, seed=40 + bps, num_blocks=600)
    o, lse = run_b200(b, blocks_per_split=bps)
    o_ref, lse_ref = run_oracle(b)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


@pytest.mark.parametrize("dtype,d", [(torch.float32, 128), (torch.bfloat16, 64), (torch.float16, 256)])
def test_long_splits_other_paths(dtype, d):
    """Splits of 48 blocks (second block id per lane) on the CUDA-core path (fp32)
    and the tensor-core path at head_dims 64 and 256."""
    b = workloads.decode_batch(5, 700, 1500, 16, 4, d, dtype, seed=77 + d, num_blocks=600)
    o, lse = run_b200(b, blocks_per_split=48)
    o_ref, lse_ref = run_oracle(b)
    assert_close(o, lse, o_ref, lse_ref, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_workspace_reuse_with_garbage(dtype):
    """The split merge needs nothing in the shared workspace to start at zero: a
    workspace full of junk, then calls of different shapes (so one call's split
    counters land on another call's partial sums) all match the oracle."""
    from serving_engine_b200 import ops
    ops.workspace(torch.device(DEV), 64 << 20).fill_(0xA5)
    shapes = [(40, 900, 32, 8), (3, 3000, 16, 2), (64, 700, 32, 8), (5, 2500, 8, 8)]
    for i, (n, ctx, hq, hkv) in enumerate(shapes):
        b = workloads.decode_batch(n, 1, ctx, hq, hkv, 128, dtype, seed=300 + i, num_blocks=n * (ctx // 16 + 2))
        o, lse = run_b200(b, blocks_per_split=2 + i)
        o_ref, lse_ref = run_oracle(b)
        assert_close(o, lse, o_ref, lse_ref, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_block_boundaries(dtype):
    lens = [1, 2, 15, 16, 17, 31, 32, 33, 47, 48, 49, 511, 512, 513]
    gen = torch.Generator().manual_seed(3)
    nb = sum(math.ceil(k / 16) for k in lens) + 5
    perm = torch.randperm(nb, generator=gen).tolist()
    tables, p = [], 0
    for k in lens:
        n = math.ceil(k / 16)
        tables.append(perm[p:p + n])
        p += n
    b = workloads.PagedBatch(q=torch.randn(len(lens), 16, 128, generator=gen).to(dtype),
                             k_cache=torch.randn(nb, 16, 4, 128, generator=gen).to(dtype),
                             v_cache=torch.randn(nb, 16, 4, 128, generator=gen).to(dtype), block_tables=tables,
                             q_lens=[1] * len(lens), k_lens=lens, q_pos_offsets=[k - 1 for k in lens],
                             num_q_heads=16, num_kv_heads=4, scale=1 / math.sqrt(128))
    for causal in (True, False):
        o, lse = run_b200(b, causal)
        o_ref, lse_ref = run_oracle(b, causal)
        assert_close(o, lse, o_ref, lse_ref, dtype)


def test_nan_pool_beyond_k_len_does_not_leak():
    """Slots of the last block past k_len may hold anything (here NaN); the
    result must not see them (the reference's loads zero-pad them)."""
    b = workloads.decode_batch(4, 1, 60, 8, 2, 128, torch.bfloat16, seed=8, num_blocks=32)
    for r, bt in enumerate(b.block_tables):
        k = b.k_lens[r]
        if k % 16:
            b.k_cache[bt[-1], k % 16:] = float("nan")
            b.v_cache[bt[-1], k % 16:] = float("nan")
    o, lse = run_b200(b)
    assert np.isfinite(o).all()
    b2 = workloads.decode_batch(4, 1, 60, 8, 2, 128, torch.bfloat16, seed=8, num_blocks=32)
    o_ref, lse_ref = run_oracle(b2)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


def test_mixed_prefill_and_decode_rows_bf16():
    """Chunked-prefill rows (q_pos_offset > 0) and decode rows in one call."""
    gen = torch.Generator().manual_seed(11)
    rows = [(64, 0), (33, 100), (1, 200), (1, 5), (17, 16)]
    nb = 64
    perm = torch.randperm(nb, generator=gen).tolist()
    tables, p = [], 0
    for ql, qp in rows:
        n = math.ceil((ql + qp) / 16)
        tables.append(perm[p:p + n])
        p += n
    tq = sum(r[0] for r in rows)
    b = workloads.PagedBatch(q=torch.randn(tq, 32, 128, generator=gen).bfloat16(),
                             k_cache=torch.randn(nb, 16, 8, 128, generator=gen).bfloat16(),
                             v_cache=torch.randn(nb, 16, 8, 128, generator=gen).bfloat16(), block_tables=tables,
                             q_lens=[r[0] for r in rows], k_lens=[sum(r) for r in rows],
                             q_pos_offsets=[r[1] for r in rows], num_q_heads=32, num_kv_heads=8,
                             scale=1 / math.sqrt(128))
    o, lse = run_b200(b)
    o_ref, lse_ref = run_oracle(b)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


def test_reference_metadata_without_extras():
    """A metadata dict with only the reference's keys (rows found on the device)."""
    b, _ = attention_batches()["mixed_fp32"]
    md = b.metadata(DEV)
    o, lse = paged_flash_attention(b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV), md, 4, 2, b.scale)
    torch.cuda.synchronize()
    check_device_errors()
    o_ref, lse_ref = run_oracle(b)
    assert_close(o.cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref, torch.float32)


def test_zero_length_row_gives_nan_and_neg_inf():
    """k_len = 0 with a query: the reference's loop never runs, O = 0/0, LSE = -inf."""
    b = workloads.decode_batch(3, 5, 40, 4, 4, 64, torch.float32, seed=2, num_blocks=16)
    b.k_lens[1] = 0
    o, lse = run_b200(b)
    assert np.isnan(o[1]).all() and np.isneginf(lse[1]).all()
    o_ref, lse_ref = run_oracle(b)
    assert_close(o[[0, 2]], lse[[0, 2]], o_ref[[0, 2]], lse_ref[[0, 2]], torch.float32)


def test_bad_block_id_reports_error_without_fault():
    b = workloads.decode_batch(2, 20, 40, 8, 2, 128, torch.bfloat16, seed=6, num_blocks=16)
    md = b.metadata(DEV)
    md["block_table"][0, 0] = 10_000
    paged_flash_attention(b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV), md, 8, 2, b.scale)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="block id out of range"):
        check_device_errors()


def test_host_validation_rejects_block_id_beyond_pool():
    b = workloads.decode_batch(2, 20, 40, 8, 2, 128, torch.bfloat16, seed=6, num_blocks=16)
    tables = [list(t) for t in b.block_tables]
    tables[1][0] = 16
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, tables, DEV)
    with pytest.raises(ValueError, match="outside the pool"):
        paged_flash_attention(b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV), md, 8, 2, b.scale)
