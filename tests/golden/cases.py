"""Seeded inputs of the golden fixtures, shared by make_golden.py and the tests.

Regenerating a case from its seed gives bit-identical tensors (torch's CPU
generator); golden.json stores their sha256 so a test can prove it.
"""
from __future__ import annotations

import hashlib

import torch

from serving_engine_b200 import workloads
from serving_engine_b200.workloads import PagedBatch


def digest(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def mixed_batch(seed: int) -> PagedBatch:
    """fp32, 4 q heads / 2 kv heads, head_dim 64: prefill chunks (one a continuation
    with q_pos_offset > 0, one sharing prefix blocks with another row) and decode
    rows whose k_len lands on and beside block boundaries."""
    gen = torch.Generator().manual_seed(seed)
    num_blocks = 40
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    # (q_len, q_pos_offset) per row; k_len = q_pos_offset + q_len
    rows = [(37, 0), (20, 45), (1, 0), (1, 15), (1, 16), (1, 32), (5, 27)]
    tables, pos = [], 0
    for ql, qp in rows:
        n = -(-(ql + qp) // 16)
        tables.append(perm[pos:pos + n])
        pos += n
    tables[6] = tables[1][:1] + tables[6][1:]  # row 6 shares row 1's first block (a prefix hit)
    total_q = sum(r[0] for r in rows)
    q = torch.randn(total_q, 4, 64, generator=gen)
    k_cache = torch.randn(num_blocks, 16, 2, 64, generator=gen)
    v_cache = torch.randn(num_blocks, 16, 2, 64, generator=gen)
    return PagedBatch(q=q, k_cache=k_cache, v_cache=v_cache, block_tables=tables,
                      q_lens=[r[0] for r in rows], k_lens=[r[0] + r[1] for r in rows],
                      q_pos_offsets=[r[1] for r in rows], num_q_heads=4, num_kv_heads=2, scale=0.125)


def attention_batches() -> dict:
    """name -> (batch, whether the Triton kernel is also run on it)."""
    return {
        "cfg1_fp32": (workloads.config1(seed=11), True),
        "gqa_bf16": (workloads.decode_batch(6, 1, 200, 8, 2, 128, torch.bfloat16, 12, num_blocks=96), False),
        "mixed_fp32": (mixed_batch(13), True),
    }


def noncausal_batch() -> PagedBatch:
    return workloads.decode_batch(5, 1, 70, 4, 4, 64, torch.float32, 14, num_blocks=32)


def kv_append_inputs(dtype: torch.dtype):
    """(pool [2, 2, 24, 16, 4, 64], k [1, 29, 4, 64], v, slots int64 [29]); layer 1 is written."""
    gen = torch.Generator().manual_seed(21)
    layers, nb, hkv, d, s = 2, 24, 4, 64, 29
    kv = torch.randn(layers, 2, nb, 16, hkv, d, generator=gen).to(dtype)
    k_src = torch.randn(1, s, hkv, d, generator=gen).to(dtype)
    v_src = torch.randn(1, s, hkv, d, generator=gen).to(dtype)
    slots = torch.randperm(nb * 16, generator=gen)[:s]
    return kv, k_src, v_src, slots


def e2e_prompts():
    """(prompts, max_new_tokens) of the end-to-end greedy-parity fixture."""
    gen = torch.Generator().manual_seed(31)
    lens = [20, 37, 5, 64]
    return [torch.randint(0, 1000, (n,), generator=gen).tolist() for n in lens], 12


def e2e_config4_workload() -> dict:
    """The end-to-end parity run on the config-4 model shape (16 layers, hidden
    2048, 32/8 heads, head_dim 64, FFN 8192, vocab 32000), reduced so the
    reference engine can run it on the CPU in fp32: 12 requests, token ids
    U[0, 32000), prompt lengths lognormal around 64 (the workload generator's
    cv = 1 spread) clipped to [20, 200], 16 greedy tokens each. Requests 3, 9
    and 11 start with request 0's first 48 tokens (three full blocks): 9 and 11
    arrive after request 0's blocks are registered and hit the prefix cache.
    8 requests arrive at step 0 and one each at steps 6, 10, 18 and 26. A
    96-token budget forces chunked prefill and mixed steps; a 20-block pool
    forces a preemption with recompute."""
    import math

    import numpy as np

    rng = np.random.default_rng(0)
    sigma = math.sqrt(math.log(2.0))
    lens = np.clip(np.round(np.exp(rng.normal(math.log(64.0), sigma, size=12))), 20, 200).astype(int)
    prompts = [rng.integers(0, 32000, size=int(k)).tolist() for k in lens]
    for j in (3, 9, 11):
        prompts[j] = prompts[0][:48] + prompts[j][:max(len(prompts[j]) - 48, 5)]
    return {"prompts": prompts, "max_new": 16, "num_gpu_blocks": 20, "max_num_batched_tokens": 96,
            "max_num_seqs": None, "min_chunk_size": None,
            "arrivals": {0: list(range(8)), 6: [8], 10: [9], 18: [10], 26: [11]}, "model": "config4", "seed": 0}
