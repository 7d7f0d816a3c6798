"""Seeded random sweep of mixed batches through the public dispatch
(paged_flash_attention: q_len == 1 rows to the split-K decode kernel, longer
rows to the tcgen05 prefill kernel, fp32 to the CUDA-core kernel) against the
fp64 oracle: random row counts, q/k lengths across block boundaries, GQA
groups, head dims, dtypes and causal / non-causal masking."""
import math

import numpy as np
import pytest
import torch

from oracle.paged_attention import paged_attention
from serving_engine_b200 import check_device_errors, paged_flash_attention, workloads
from serving_engine_b200.paged_attention import metadata_from_lists
from tests.test_paged_decode_gpu import assert_close

pytestmark = pytest.mark.gpu
HEADS = [(32, 8), (8, 8), (16, 4), (32, 4), (16, 1), (12, 12), (16, 2)]


def random_batch(rng, hq, hkv, d, dtype):
    rows = []
    for _ in range(int(rng.integers(1, 7))):
        q_len = 1 if rng.random() < 0.5 else int(rng.integers(2, 300))
        q_pos = int(rng.integers(0, 1500))
        if rng.random() < 0.2:  # land the row's end on a block boundary
            q_pos = max(0, 16 * ((q_pos + q_len) // 16 + 1) - q_len)
        rows.append((q_len, q_pos))
    need = [math.ceil((ql + qp) / 16) for ql, qp in rows]
    nb = sum(need) + int(rng.integers(1, 10))
    gen = torch.Generator().manual_seed(int(rng.integers(0, 2**31)))
    perm = torch.randperm(nb, generator=gen).tolist()
    tables, p = [], 0
    for n in need:
        tables.append(perm[p:p + n])
        p += n
    tq = sum(r[0] for r in rows)
    return workloads.PagedBatch(q=torch.randn(tq, hq, d, generator=gen).to(dtype),
                                k_cache=torch.randn(nb, 16, hkv, d, generator=gen).to(dtype),
                                v_cache=torch.randn(nb, 16, hkv, d, generator=gen).to(dtype), block_tables=tables,
                                q_lens=[r[0] for r in rows], k_lens=[sum(r) for r in rows],
                                q_pos_offsets=[r[1] for r in rows], num_q_heads=hq, num_kv_heads=hkv,
                                scale=1 / math.sqrt(d))


@pytest.mark.parametrize("case", range(24))
def test_random_mixed_batch_matches_oracle(case):
    rng = np.random.default_rng(1000 + case)
    dtype = torch.float32 if case % 6 == 5 else (torch.bfloat16 if case % 2 == 0 else torch.float16)
    hq, hkv = HEADS[int(rng.integers(0, len(HEADS)))]
    d = 64 if rng.random() < 0.5 else 128
    causal = case % 5 != 4
    b = random_batch(rng, hq, hkv, d, dtype)
    md = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, "cuda")
    o, lse = paged_flash_attention(b.q.cuda(), b.k_cache.cuda(), b.v_cache.cuda(), md, hq, hkv, b.scale, causal)
    torch.cuda.synchronize()
    check_device_errors()
    mdc = b.metadata("cpu")
    o_ref, lse_ref = paged_attention(b.q, b.k_cache, b.v_cache, mdc["block_table"], mdc["q_starts"], mdc["q_lens"],
                                     mdc["k_lens"], mdc["q_pos_offsets"], b.scale, causal)
    assert_close(o.float().cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref, dtype)
