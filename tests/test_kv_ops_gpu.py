"""KV append and copy-on-write block copy on the GPU: bit-exact against the
reference semantics (index_copy_ / fancy-index assignment) and the oracle."""
import numpy as np
import pytest
import torch

from oracle import kv_ops
from serving_engine_b200 import PagedKVCache, check_device_errors, copy_blocks, kv_append, workloads
from tests.golden.cases import digest, kv_append_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("tag,dtype", [("fp32", torch.float32), ("bf16", torch.bfloat16)])
def test_kv_append_matches_golden(tag, dtype, golden_arrays, golden_meta):
    kv, k_src, v_src, slots = kv_append_inputs(dtype)
    meta = golden_meta[f"kv_append_{tag}"]
    pool = kv.to(DEV)
    cache = PagedKVCache(pool)
    # HF hands [1, HKV, S, D] views that are transposes of [1, S, HKV, D] storage
    cache.write(k_src.to(DEV).transpose(1, 2), v_src.to(DEV).transpose(1, 2), 1, slots.to(DEV))
    check_device_errors()
    assert digest(pool) == meta["pool_after"]
    written = pool[1].reshape(2, -1, 4, 64)[:, slots.to(DEV)].float().cpu().numpy()
    np.testing.assert_array_equal(written, golden_arrays[f"kv_append_{tag}__written"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_kv_append_config3_scale_bit_exact(dtype):
    """Config-3 append: 16 x 512 new tokens scattered into fresh blocks."""
    b = workloads.config3(seed=3)
    kc = b.k_cache.to(DEV, dtype)
    vc = b.v_cache.to(DEV, dtype)
    nk = b.extra["new_k"].to(DEV, dtype)
    nv = b.extra["new_v"].to(DEV, dtype)
    slots = b.extra["slot_mapping"].to(DEV)
    ref_k, ref_v = kc.clone(), vc.clone()
    ref_k.view(-1, 8, 128).index_copy_(0, slots, nk)
    ref_v.view(-1, 8, 128).index_copy_(0, slots, nv)
    kv_append(nk, nv, kc, vc, slots)
    check_device_errors()
    assert torch.equal(kc.view(torch.int8), ref_k.view(torch.int8))
    assert torch.equal(vc.view(torch.int8), ref_v.view(torch.int8))


def test_kv_append_matches_oracle_strided_and_odd_strides():
    gen = torch.Generator().manual_seed(5)
    nb, h, d, n = 12, 3, 64, 40
    kc = torch.randn(nb, 16, h, d, generator=gen)
    vc = torch.randn(nb, 16, h, d, generator=gen)
    # source with an odd token stride (vector width falls back below 16 bytes)
    big = torch.randn(n, h * d + 1, generator=gen)
    k_new = torch.as_strided(big, (n, h, d), (h * d + 1, d, 1))
    v_new = torch.randn(n, h, d, generator=gen)
    slots = torch.randperm(nb * 16, generator=gen)[:n]
    ko, vo = kc.numpy().copy(), vc.numpy().copy()
    kv_ops.kv_append(ko, vo, k_new.numpy(), v_new.numpy(), slots.numpy())
    kc_d, vc_d = kc.to(DEV), vc.to(DEV)
    kv_append(torch.as_strided(big.to(DEV), (n, h, d), (h * d + 1, d, 1)), v_new.to(DEV), kc_d, vc_d, slots.to(DEV))
    check_device_errors()
    np.testing.assert_array_equal(kc_d.cpu().numpy(), ko)
    np.testing.assert_array_equal(vc_d.cpu().numpy(), vo)


def test_kv_append_out_of_range_slot_sets_error_and_skips():
    kc = torch.zeros(4, 16, 2, 64, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    new = torch.ones(3, 2, 64, device=DEV, dtype=torch.bfloat16)
    slots = torch.tensor([5, 64, -1], device=DEV, dtype=torch.int64)
    kv_append(new, new, kc, vc, slots)
    with pytest.raises(RuntimeError, match="slot out of range"):
        check_device_errors()
    flat = kc.view(-1, 2, 64)
    assert torch.all(flat[5] == 1) and int((flat != 0).sum()) == 2 * 64
    check_device_errors()  # the word was reset


def test_kv_append_empty_and_validation():
    kc = torch.zeros(4, 16, 2, 64, device=DEV)
    kv_append(torch.empty(0, 2, 64, device=DEV), torch.empty(0, 2, 64, device=DEV), kc, kc.clone(),
              torch.empty(0, dtype=torch.int64, device=DEV))
    with pytest.raises(ValueError):
        kv_append(torch.zeros(2, 2, 64, device=DEV), torch.zeros(2, 2, 64, device=DEV), kc, kc.clone(),
                  torch.zeros(2, dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError):
        kv_append(torch.zeros(2, 2, 64, device=DEV, dtype=torch.bfloat16),
                  torch.zeros(2, 2, 64, device=DEV, dtype=torch.bfloat16), kc, kc.clone(),
                  torch.zeros(2, dtype=torch.int64, device=DEV))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_copy_blocks_matches_oracle(dtype):
    gen = torch.Generator().manual_seed(9)
    pool = torch.randn(3, 2, 20, 16, 4, 64, generator=gen).to(dtype)
    src, dst = [2, 5, 5, 11], [17, 3, 19, 0]
    ref = pool.clone()
    ref_np = ref.view(torch.int16).numpy() if dtype == torch.bfloat16 else ref.numpy()
    kv_ops.copy_blocks(ref_np, src, dst)
    dpool = pool.to(DEV)
    PagedKVCache(dpool).copy_blocks(src, dst)
    check_device_errors()
    assert torch.equal(dpool.cpu().view(torch.int8), ref.view(torch.int8))


def test_copy_blocks_config3_cow():
    """Config-3 CoW: the partially filled last prefix block (2040-token prefix) copied
    into each of 16 sequences' first private block, all layers, K and V."""
    b = workloads.config3(seed=4, prefix_len=2040)
    assert len(b.extra["cow_dst"]) == 16
    layers = 4
    pool = torch.randn(layers, 2, b.k_cache.shape[0], 16, 8, 128, device=DEV).to(torch.bfloat16)
    ref = pool.clone()
    ref[:, :, b.extra["cow_dst"]] = ref[:, :, b.extra["cow_src"]]
    copy_blocks(pool, b.extra["cow_src"], b.extra["cow_dst"])
    check_device_errors()
    assert torch.equal(pool.view(torch.int16), ref.view(torch.int16))


def test_copy_blocks_validation_and_errors():
    pool = torch.zeros(1, 2, 8, 16, 2, 64, device=DEV)
    with pytest.raises(ValueError, match="duplicate"):
        copy_blocks(pool, [1, 2], [3, 3])
    with pytest.raises(ValueError, match="also a src"):
        copy_blocks(pool, [1, 2], [2, 4])
    with pytest.raises(ValueError, match="out of range"):
        copy_blocks(pool, [1], [8])
    copy_blocks(pool, [], [])
    # device-tensor ids skip host validation; the kernel flags and skips bad ids
    copy_blocks(pool, torch.tensor([1, 9], device=DEV), torch.tensor([2, 3], device=DEV))
    with pytest.raises(RuntimeError, match="block id out of range"):
        check_device_errors()
