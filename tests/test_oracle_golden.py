"""Pin the CPU oracle to outputs of the reference itself (tests/golden/).

The fixtures were produced by tests/golden/make_golden.py running the
reference's eager oracle path, its Triton kernel (interpreted), its
index_copy_ KV write and its metadata builder on seeded inputs; these tests
regenerate the inputs, prove they are bit-identical (sha256) and check each
oracle function against the recorded outputs.
"""
import numpy as np
import pytest
import torch

from oracle import kv_ops
from oracle.paged_attention import paged_attention
from serving_engine_b200.paged_attention import metadata_from_lists
from tests.golden.cases import attention_batches, digest, kv_append_inputs, noncausal_batch


def _oracle(b, causal=True):
    md = b.metadata("cpu")
    return paged_attention(b.q, b.k_cache, b.v_cache, md["block_table"], md["q_starts"], md["q_lens"],
                           md["k_lens"], md["q_pos_offsets"], b.scale, causal)


@pytest.mark.parametrize("name", ["cfg1_fp32", "gqa_bf16", "mixed_fp32"])
def test_inputs_regenerate_bit_identical(name, golden_meta):
    b, _ = attention_batches()[name]
    assert digest(b.q) == golden_meta[name]["q"]
    assert digest(b.k_cache) == golden_meta[name]["k_cache"]
    assert digest(b.v_cache) == golden_meta[name]["v_cache"]


@pytest.mark.parametrize("name", ["cfg1_fp32", "mixed_fp32"])
def test_oracle_matches_reference_fp32(name, golden_arrays):
    """fp32: oracle vs the reference eager path and vs its Triton kernel (o and LSE)."""
    b, _ = attention_batches()[name]
    o, lse = _oracle(b)
    np.testing.assert_allclose(o, golden_arrays[f"{name}__eager"], atol=1e-5, rtol=0)
    np.testing.assert_allclose(o, golden_arrays[f"{name}__triton_o"], atol=1e-5, rtol=0)
    np.testing.assert_allclose(lse, golden_arrays[f"{name}__triton_lse"], atol=1e-5, rtol=0)


def test_oracle_matches_reference_bf16(golden_arrays):
    """bf16 inputs: the oracle (fp64 on the bf16 values) equals the reference eager path
    run in fp32 on the same values; the reference's own bf16 eager output (scores and
    probabilities rounded to bf16) stays within its documented drift."""
    b, _ = attention_batches()["gqa_bf16"]
    o, _ = _oracle(b)
    np.testing.assert_allclose(o, golden_arrays["gqa_bf16__eager_fp32"], atol=1e-5, rtol=0)
    assert np.abs(o - golden_arrays["gqa_bf16__eager"]).max() < 3e-2


def test_oracle_noncausal_matches_triton(golden_arrays, golden_meta):
    b = noncausal_batch()
    assert digest(b.q) == golden_meta["noncausal_fp32"]["q"]
    o, lse = _oracle(b, causal=False)
    np.testing.assert_allclose(o, golden_arrays["noncausal_fp32__triton_o"], atol=1e-5, rtol=0)
    np.testing.assert_allclose(lse, golden_arrays["noncausal_fp32__triton_lse"], atol=1e-5, rtol=0)


def test_noncausal_differs_from_exclusion_on_partial_blocks():
    """The zero-padded keys of a partial last block enter a non-causal softmax with
    score 0 in the reference kernel; a plain 'drop keys past k_len' would differ."""
    b = noncausal_batch()
    assert any(k % 16 for k in b.k_lens)
    o_nc, _ = _oracle(b, causal=False)
    o_c, _ = _oracle(b, causal=True)  # decode rows: causal == exactly the real keys
    assert np.abs(o_nc - o_c).max() > 1e-3


@pytest.mark.parametrize("tag,dtype", [("fp32", torch.float32), ("bf16", torch.bfloat16)])
def test_oracle_kv_append_matches_index_copy(tag, dtype, golden_arrays, golden_meta):
    kv, k_src, v_src, slots = kv_append_inputs(dtype)
    meta = golden_meta[f"kv_append_{tag}"]
    assert digest(kv) == meta["kv"] and slots.tolist() == meta["slots"]
    pool = kv.clone()
    view = pool.view(torch.int16) if dtype == torch.bfloat16 else pool
    arr = view.numpy()
    src_k = (k_src.view(torch.int16) if dtype == torch.bfloat16 else k_src)[0].numpy()
    src_v = (v_src.view(torch.int16) if dtype == torch.bfloat16 else v_src)[0].numpy()
    kv_ops.kv_append(arr[1, 0], arr[1, 1], src_k, src_v, slots.numpy())
    assert digest(pool) == meta["pool_after"]
    written = pool[1].reshape(2, -1, *pool.shape[-2:])[:, slots].float().numpy()
    np.testing.assert_array_equal(written, golden_arrays[f"kv_append_{tag}__written"])


def test_oracle_copy_blocks_semantics():
    rng = np.random.default_rng(0)
    pool = rng.standard_normal((3, 2, 10, 16, 2, 8)).astype(np.float32)
    ref = pool.copy()
    src, dst = [1, 4, 4], [7, 2, 9]
    kv_ops.copy_blocks(pool, src, dst)
    for s, d in zip(src, dst):
        np.testing.assert_array_equal(pool[:, :, d], ref[:, :, s])
    untouched = [b for b in range(10) if b not in dst]
    np.testing.assert_array_equal(pool[:, :, untouched], ref[:, :, untouched])


def test_oracle_metadata_matches_reference_trace(golden_meta):
    steps = golden_meta["scheduler_trace"]
    assert len(steps) >= 10
    kinds = {r["phase"] for s in steps for r in s["rows"]}
    assert kinds == {"NEEDS_PREFILL", "NEEDS_DECODE"}
    for s in steps:
        md = kv_ops.build_metadata(s["rows"])
        assert md == s["metadata"]
        assert kv_ops.write_indices(s["rows"]) == s["write_index"]


def test_package_metadata_builder_matches_reference_trace(golden_meta):
    """serving_engine_b200.build_paged_batch_metadata's reference keys equal the
    reference builder's output at every step of the scripted scheduler run."""
    from types import SimpleNamespace

    from serving_engine_b200 import build_paged_batch_metadata

    for s in golden_meta["scheduler_trace"]:
        reqs, chunks = [], {}
        for i, r in enumerate(s["rows"]):
            rid = f"q{i}"
            prompt_len = r["total_len"]
            reqs.append(SimpleNamespace(request_id=rid, phase=SimpleNamespace(name=r["phase"]),
                                        num_computed_tokens=r["num_computed_tokens"], total_len=prompt_len,
                                        block_table=r["block_table"]))
            chunks[rid] = r["chunk"]
        so = SimpleNamespace(scheduled_requests=reqs, prefill_chunk_sizes=chunks)
        md = build_paged_batch_metadata(so, device="cpu")
        ref = s["metadata"]
        for k in ("q_lens", "k_lens", "q_starts", "q_pos_offsets", "block_table"):
            assert md[k].dtype == torch.int32
            assert md[k].tolist() == ref[k], k
        assert md["block_table_row_stride"] == ref["block_table_row_stride"]
        assert md["total_query"] == ref["total_query"]
        # extras: per-token row ids and host maxima
        rows = [r for r, n in enumerate(ref["q_lens"]) for _ in range(n)]
        assert md["item_row"].tolist() == rows
        assert md["max_q_len"] == max(ref["q_lens"])


def test_metadata_from_lists_empty():
    md = metadata_from_lists([], [], [], [], [], "cpu")
    assert md["total_query"] == 0 and md["block_table"].shape == (0, 0) and md["max_q_len"] == 0
