"""Mixed batches described only by the reference builder's dict keys
(q_lens, k_lens, q_starts, q_pos_offsets, block_table, block_table_row_stride,
total_query: what build_paged_batch_metadata in
serving_engine/paged_attention_kernel.py:163-200 returns and ModelRunner.forward
passes on at model_runner.py:184). paged_flash_attention routes their rows on
the device: q_len > 1 rows must reach the tcgen05 prefill kernel (seen in the
kernel launches the profiler records), q_len == 1 rows the split-K decode
kernel, and the result must match the CPU oracle."""
import math

import numpy as np
import pytest
import torch
from torch.profiler import ProfilerActivity, profile

from oracle.paged_attention import paged_attention
from serving_engine_b200 import check_device_errors, ops, paged_flash_attention, workloads
from tests.test_paged_decode_gpu import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_batch(rows, hq, hkv, d, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    need = [math.ceil((ql + qp) / 16) for ql, qp in rows]
    nb = sum(need) + 5
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


def kernels_launched(fn):
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        out = fn()
        torch.cuda.synchronize()
    names = {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}
    return out, names


def oracle(b, is_causal=True):
    md = b.metadata("cpu")
    return paged_attention(b.q, b.k_cache, b.v_cache, md["block_table"], md["q_starts"], md["q_lens"], md["k_lens"],
                           md["q_pos_offsets"], b.scale, is_causal)


@pytest.mark.parametrize("d,hq,hkv", [(128, 32, 8), (64, 32, 8), (128, 16, 16), (64, 8, 2)])
def test_reference_dict_reaches_the_prefill_kernel(d, hq, hkv):
    rows = [(1, 700), (600, 0), (1, 31), (257, 1024), (1, 2047), (40, 5), (1, 0)]
    b = make_batch(rows, hq, hkv, d, torch.bfloat16, seed=d + hq)
    md = b.metadata(DEV)  # reference keys only: no host-side row split
    assert "prefill_rows" not in md and "item_row" not in md
    q, kc, vc = b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV)
    launches = ops.LAUNCHES[0]
    (o, lse), names = kernels_launched(lambda: paged_flash_attention(q, kc, vc, md, hq, hkv, b.scale))
    check_device_errors()
    assert ops.LAUNCHES[0] - launches == 3
    assert any("route_rows_kernel" in n for n in names), names
    assert any("decode_mma_kernel" in n for n in names), names
    prefill = "prefill_pair_kernel" if d == 128 else "prefill_tc_kernel"
    assert any(prefill in n for n in names), names
    o_ref, lse_ref = oracle(b)
    assert_close(o.float().cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref, torch.bfloat16)


def test_reference_dict_many_rows_and_chunks():
    """More rows than one routing pass of 1024 threads, decode rows and prefill
    rows interleaved; fp16; non-causal too."""
    rng = np.random.default_rng(5)
    rows = []
    for i in range(1500):
        if i % 97 == 3:
            rows.append((int(rng.integers(2, 200)), int(rng.integers(0, 300))))
        else:
            rows.append((1, int(rng.integers(0, 400))))
    b = make_batch(rows, 16, 4, 128, torch.float16, seed=3)
    md = b.metadata(DEV)
    q, kc, vc = b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV)
    for causal in (True, False):
        o, lse = paged_flash_attention(q, kc, vc, md, 16, 4, b.scale, causal)
        torch.cuda.synchronize()
        check_device_errors()
        o_ref, lse_ref = oracle(b, causal)
        assert_close(o.float().cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref, torch.float16)


def test_reference_dict_matches_host_split_bitwise():
    """The device-routed call and the host-split call run the same kernels on the
    same work: identical outputs."""
    from serving_engine_b200.paged_attention import metadata_from_lists

    rows = [(130, 300), (1, 999), (77, 0), (1, 64), (512, 2040)]
    b = make_batch(rows, 32, 8, 128, torch.bfloat16, seed=77)
    q, kc, vc = b.q.to(DEV), b.k_cache.to(DEV), b.v_cache.to(DEV)
    o1, l1 = paged_flash_attention(q, kc, vc, b.metadata(DEV), 32, 8, b.scale)
    md2 = metadata_from_lists(b.q_lens, b.k_lens, b.q_starts, b.q_pos_offsets, b.block_tables, DEV)
    o2, l2 = paged_flash_attention(q, kc, vc, md2, 32, 8, b.scale)
    torch.cuda.synchronize()
    check_device_errors()
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    assert torch.equal(l1, l2)
