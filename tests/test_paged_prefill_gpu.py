"""Chunked-prefill paged attention on tcgen05 tensor cores (through the C ABI)
against the CPU oracle, and the q_len-based dispatch of paged_flash_attention.

Tolerance (tests/tolerance.py): bf16/fp16 O within 2e-3 of the fp64 oracle on
the same 16-bit values where half an ulp of the stored type is <= 1e-3 (bf16:
|O| < 0.5), plus half an ulp of the reference value above that; LSE within 1e-3.
"""
import math

import numpy as np
import pytest
import torch

from oracle.paged_attention import paged_attention
from serving_engine_b200 import check_device_errors, ops, paged_flash_attention, workloads
from serving_engine_b200.paged_attention import metadata_from_lists
from tests.test_paged_decode_gpu import assert_close, assert_out_close
from tests.tolerance import band_report, strict_mask

pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_batch(rows, hq, hkv, d, dtype, seed, shared_prefix_blocks=0, nan_tail=False):
    """rows: list of (q_len, q_pos_offset); k_len = q_pos_offset + q_len."""
    gen = torch.Generator().manual_seed(seed)
    need = [math.ceil((ql + qp) / 16) for ql, qp in rows]
    nb = sum(need) + 8
    perm = torch.randperm(nb, generator=gen).tolist()
    tables, p = [], 0
    for n in need:
        tables.append(perm[p:p + n])
        p += n
    if shared_prefix_blocks:
        for t in tables[1:]:
            k = min(shared_prefix_blocks, len(t) - 1, len(tables[0]) - 1)
            t[:k] = tables[0][:k]
    tq = sum(r[0] for r in rows)
    b = workloads.PagedBatch(q=torch.randn(tq, hq, d, generator=gen).to(dtype),
                             k_cache=torch.randn(nb, 16, hkv, d, generator=gen).to(dtype),
                             v_cache=torch.randn(nb, 16, hkv, d, generator=gen).to(dtype), block_tables=tables,
                             q_lens=[r[0] for r in rows], k_lens=[sum(r) for r in rows],
                             q_pos_offsets=[r[1] for r in rows], num_q_heads=hq, num_kv_heads=hkv,
                             scale=1 / math.sqrt(d))
    if nan_tail:
        for r, t in enumerate(tables):
            k = b.k_lens[r]
            if k % 16:
                b.k_cache[t[(k - 1) // 16], k % 16:] = float("nan")
                b.v_cache[t[(k - 1) // 16], k % 16:] = float("nan")
    return b


def run_prefill(b, is_causal=True):
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, DEV)
    o, lse = ops.paged_prefill(b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV), md["block_table"], md["q_starts"],
                               md["q_lens"], md["k_lens"], md["q_pos_offsets"], b.num_q_heads, b.num_kv_heads, b.scale,
                               is_causal, max_q_len=max(b.q_lens))
    torch.cuda.synchronize()
    check_device_errors()
    return o.float().cpu().numpy(), lse.cpu().numpy()


def oracle(b, is_causal=True, **kw):
    md = b.metadata("cpu")
    return paged_attention(b.q, b.k_cache, b.v_cache, md["block_table"], md["q_starts"], md["q_lens"], md["k_lens"],
                           md["q_pos_offsets"], b.scale, is_causal, **kw)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (16, 8), (32, 4), (16, 1)])
@pytest.mark.parametrize("d", [64, 128])
def test_prefill_shapes_vs_oracle(dtype, hq, hkv, d):
    rows = [(70, 0), (33, 100), (128, 37), (5, 300)]
    b = make_batch(rows, hq, hkv, d, dtype, seed=hq + hkv * 3 + d)
    o, lse = run_prefill(b)
    o_ref, lse_ref = oracle(b)
    assert_close(o, lse, o_ref, lse_ref, dtype)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (32, 4), (16, 1)])
@pytest.mark.parametrize("d", [64, 128])
def test_prefill_q_tile_pairs(hq, hkv, d):
    """A CTA computes a pair of Q tiles of 128 // group queries each. Rows whose
    second tile holds a single query or a ragged tail, pairs that run as two CTAs
    (early positions, P's remainder) next to pairs that run as one, and a row
    crossing from the first kind to the second all match the oracle."""
    qpt = 128 // (hq // hkv)
    rows = [(qpt + 1, 300), (2 * qpt + 1, 400), (3 * qpt - 5, 260), (300, 100), (2 * qpt, 1000)]
    b = make_batch(rows, hq, hkv, d, torch.bfloat16, seed=17 + hq + d)
    o, lse = run_prefill(b)
    o_ref, lse_ref = oracle(b)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


def test_prefill_long_chunk_shared_prefix():
    """Config-3 pattern at reduced size: rows share prefix blocks, then prefill a chunk."""
    rows = [(200, 512)] * 4
    b = make_batch(rows, 32, 8, 128, torch.bfloat16, seed=5, shared_prefix_blocks=32)
    o, lse = run_prefill(b)
    o_ref, lse_ref = oracle(b)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (32, 4), (16, 1)])
def test_prefill_long_context_rows(hq, hkv):
    """Pairs whose first query sees at least 1,024 keys skip P's remainder pass;
    on their unmasked tiles part of the exponentials is a polynomial on the FMA
    pipe instead of the MUFU's ex2. Ragged tails, partial last blocks and a
    row that crosses from split pairs to unsplit ones meet the same bound, the
    plain 2e-3 where it applies included."""
    rows = [(96, 1100), (130, 2047), (33, 1500), (200, 900)]
    b = make_batch(rows, hq, hkv, 128, torch.bfloat16, seed=41 + hq + hkv)
    o, lse = run_prefill(b)
    o_ref, lse_ref = oracle(b)
    strict = strict_mask(o_ref, torch.bfloat16)
    worst = float(np.abs(o - o_ref)[strict].max())
    assert worst <= 2e-3, f"strict band max error {worst:.3g}; bands {band_report(o, o_ref)}"
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_nan_key_poisons_the_rows_that_see_it(d):
    """A NaN in a visible key makes every output (and LSE) of the query heads
    that see it NaN, as the reference's exp of a NaN score does, whichever way
    the exponential was evaluated; queries that do not see it, other kv heads
    and other rows stay finite and match the oracle."""
    rows = [(64, 1200), (40, 1300), (80, 600)]
    b = make_batch(rows, 32, 8, d, torch.bfloat16, seed=31 + d)
    key = 1210  # inside row 0's chunk: its first 10 queries do not see it
    b.k_cache[b.block_tables[0][key // 16], key % 16, 3, 5] = float("nan")
    o, lse = run_prefill(b)
    o_ref, lse_ref = oracle(b)
    assert np.isnan(o_ref[10:64, 12:16]).all() and not np.isnan(o_ref[:10]).any()
    assert not np.isnan(np.delete(o_ref[:64], range(12, 16), axis=1)).any() and not np.isnan(o_ref[64:]).any()
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("scale_mul", [-1.0, 0.0, 0.5])
def test_prefill_any_scale(d, scale_mul):
    """The kernels fold a positive scale into the row max and the exponent;
    a negative or zero scale (legal for the reference, which just multiplies)
    takes the path that scales scores first, and still matches the oracle."""
    rows = [(70, 1100), (33, 0), (130, 200)]
    b = make_batch(rows, 32, 8, d, torch.bfloat16, seed=53 + d)
    b.scale = scale_mul / math.sqrt(d)
    o, lse = run_prefill(b)
    o_ref, lse_ref = oracle(b)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


def test_prefill_noncausal_and_partial_blocks():
    rows = [(40, 0), (17, 9), (64, 63)]
    b = make_batch(rows, 16, 4, 128, torch.bfloat16, seed=7)
    o, lse = run_prefill(b, is_causal=False)
    o_ref, lse_ref = oracle(b, is_causal=False)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


def test_prefill_nan_pool_tail_does_not_leak():
    rows = [(45, 3), (30, 50)]
    b = make_batch(rows, 32, 8, 128, torch.bfloat16, seed=9, nan_tail=True)
    o, lse = run_prefill(b)
    assert np.isfinite(o).all()
    clean = make_batch(rows, 32, 8, 128, torch.bfloat16, seed=9)
    o_ref, lse_ref = oracle(clean)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)


def test_config3_full_size_sampled():
    """Full config 3: 16 rows x 512-token chunks after a shared 2048-token prefix,
    32/8 heads, D=128; two rows x one GQA group checked against the oracle, all
    outputs finite."""
    b = workloads.config3(seed=1)
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, DEV)
    o, lse = ops.paged_prefill(b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV), md["block_table"], md["q_starts"],
                               md["q_lens"], md["k_lens"], md["q_pos_offsets"], 32, 8, b.scale, True,
                               max_q_len=512)
    torch.cuda.synchronize()
    check_device_errors()
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    heads = [4, 5, 6, 7]
    o_ref, lse_ref = oracle(b, rows=[0, 11], heads=heads)
    for r in (0, 11):
        sl = slice(r * 512, (r + 1) * 512)
        assert_out_close(o[sl][:, heads].float().cpu().numpy(), o_ref[sl][:, heads], torch.bfloat16)
        np.testing.assert_allclose(lse[sl][:, heads].cpu().numpy(), lse_ref[sl][:, heads], atol=1e-3, rtol=0)


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_persistent_walk_vs_oracle(d):
    """More units than resident CTAs (560 real units of 1,120 named; 148 CTAs at
    head_dim 64, 74 CTA pairs at 128), so each CTA walks several units with its
    Q buffers, K/V rings and barrier phases running on from unit to unit: units
    of one and of two Q tiles, with and without the P-remainder pass, short and
    long key ranges. The host-split launch and the device router's unit list
    both match the oracle, and each other bit for bit (a unit's arithmetic does
    not depend on the CTA that runs it or on what that CTA ran before)."""
    pattern = [(33, 0), (64, 5), (65, 300), (7, 1500), (130, 0), (200, 64), (96, 1100)]
    rows = [pattern[i % len(pattern)] for i in range(35)]
    b = make_batch(rows, 32, 8, d, torch.bfloat16, seed=91 + d)
    o_ref, lse_ref = oracle(b)
    o, lse = run_prefill(b)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, DEV)
    o2, lse2 = paged_flash_attention(b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV), md, 32, 8, b.scale)
    torch.cuda.synchronize()
    check_device_errors()
    o2 = o2.float().cpu().numpy()
    lse2 = lse2.cpu().numpy()
    assert_close(o2, lse2, o_ref, lse_ref, torch.bfloat16)
    np.testing.assert_array_equal(o2, o)
    np.testing.assert_array_equal(lse2, lse)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("fault", ["k_len", "row"])
def test_prefill_metadata_errors_reported_without_fault(d, fault):
    """Host-split launches check their metadata on the device, beside the first
    loads: a k_len needing more blocks than its block-table row holds sets the
    k_len bit, a listed row index outside the batch the index bit. Nothing
    faults, and the rows with good metadata match the oracle."""
    rows = [(70, 0), (33, 100), (128, 37)]
    b = make_batch(rows, 32, 8, d, torch.bfloat16, seed=5 + d)
    o_ref, lse_ref = oracle(b)
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, DEV)
    k_lens = md["k_lens"].clone()
    listed = None
    if fault == "k_len":
        # one block past row 0's table row; its causal queries see none of it
        k_lens[0] = 16 * md["block_table"].shape[1] + 16
        match = "k_len exceeds block table row"
    else:
        listed = torch.tensor([1, 2, 7], dtype=torch.int32, device=DEV)  # row 7 is not in the batch
        match = "row/query index out of range"
    o, lse = ops.paged_prefill(b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV), md["block_table"], md["q_starts"],
                               md["q_lens"], k_lens, md["q_pos_offsets"], 32, 8, b.scale, True,
                               max_q_len=max(b.q_lens), rows=listed)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match=match):
        check_device_errors()
    sl = slice(b.q_starts[1], b.q_starts[2] + b.q_lens[2])  # rows 1 and 2
    assert_close(o.float().cpu().numpy()[sl], lse.cpu().numpy()[sl], o_ref[sl], lse_ref[sl], torch.bfloat16)


def test_dispatch_mixed_decode_and_prefill_rows():
    """paged_flash_attention sends q_len == 1 rows to the decode kernel and
    q_len > 1 rows to the tcgen05 prefill kernel; together they match the oracle."""
    rows = [(1, 300), (77, 0), (1, 15), (130, 900), (1, 0), (16, 16)]
    b = make_batch(rows, 32, 8, 128, torch.bfloat16, seed=13)
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, DEV)
    assert md["decode_tokens"].numel() == 3 and md["prefill_rows"].numel() == 3
    launches = ops.LAUNCHES[0]
    o, lse = paged_flash_attention(b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV), md, 32, 8, b.scale)
    torch.cuda.synchronize()
    check_device_errors()
    assert ops.LAUNCHES[0] - launches >= 2
    o_ref, lse_ref = oracle(b)
    assert_close(o.float().cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref, torch.bfloat16)


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_error_per_magnitude_band(d):
    """Fresh prompts (the early positions, where few keys are visible and the
    P-remainder pass runs) next to long continuations: the largest error where
    the plain 2e-3 applies (|O| < 0.5 in bf16) stays within it, and the report
    per |O| band shows how much of the rest is the output's own rounding."""
    rows = [(300, 0), (128, 0), (77, 0), (200, 700), (64, 2000)]
    b = make_batch(rows, 32, 8, d, torch.bfloat16, seed=23 + d)
    o, lse = run_prefill(b)
    o_ref, lse_ref = oracle(b)
    report = band_report(o, o_ref)
    strict = strict_mask(o_ref, torch.bfloat16)
    worst = float(np.abs(o - o_ref)[strict].max())
    assert worst <= 2e-3, f"strict band max error {worst:.3g}; bands {report}"
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)
