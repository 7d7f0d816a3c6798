"""Restatements of the reference's KV write, block copy and metadata builder
(TEST INFRASTRUCTURE ONLY).
"""
from __future__ import annotations

import numpy as np

BLOCK_SIZE = 16


def kv_append(k_cache: np.ndarray, v_cache: np.ndarray, k_new: np.ndarray, v_new: np.ndarray, slots) -> None:
    """_PagedKVCache.write (serving_engine/model_runner.py:21-32): the pool's flat
    [num_blocks*16, HKV, D] view gets row t of the new K/V at slot slots[t]
    (index_copy_ along dim 0). In place on numpy arrays."""
    kf = k_cache.reshape(-1, *k_cache.shape[2:])
    vf = v_cache.reshape(-1, *v_cache.shape[2:])
    slots = np.asarray(slots, dtype=np.int64)
    kf[slots] = k_new
    vf[slots] = v_new


def flat_slot(block_table, logical_pos: int, block_size: int = BLOCK_SIZE) -> int:
    """ModelRunner._flat_slot (serving_engine/model_runner.py:127-129)."""
    return block_table[logical_pos // block_size] * block_size + logical_pos % block_size


def copy_blocks(kv_cache: np.ndarray, src, dst) -> None:
    """kv_cache[:, :, dst] = kv_cache[:, :, src] on the engine pool
    [L, 2, num_blocks, 16, HKV, D] (model_runner.py:101-110). The sources are read
    before any destination is written (numpy fancy-index semantics)."""
    src = np.asarray(src, dtype=np.int64)
    dst = np.asarray(dst, dtype=np.int64)
    kv_cache[:, :, dst] = kv_cache[:, :, src].copy()


def build_metadata(rows) -> dict:
    """build_paged_batch_metadata (serving_engine/paged_attention_kernel.py:163-200)
    on plain data. `rows` is a list of dicts with keys phase ("NEEDS_PREFILL" or
    "NEEDS_DECODE"), chunk (prefill chunk size), num_computed_tokens, total_len,
    block_table. Returns python lists under the reference's keys."""
    q_lens, k_lens, q_starts, q_pos_offsets, tables = [], [], [], [], []
    start = 0
    for r in rows:
        if r["phase"] == "NEEDS_PREFILL":
            nq = r["chunk"]
            nk = r["num_computed_tokens"] + nq
            qp = r["num_computed_tokens"]
        else:
            nq = 1
            nk = r["total_len"]
            qp = r["total_len"] - 1
        q_lens.append(nq)
        k_lens.append(nk)
        q_starts.append(start)
        q_pos_offsets.append(qp)
        tables.append(list(r["block_table"]))
        start += nq
    width = max((len(t) for t in tables), default=0)
    return {
        "q_lens": q_lens,
        "k_lens": k_lens,
        "q_starts": q_starts,
        "q_pos_offsets": q_pos_offsets,
        "block_table": [t + [0] * (width - len(t)) for t in tables],
        "block_table_row_stride": width,
        "total_query": start,
    }


def write_indices(rows) -> list[int]:
    """Per new token, the flat slot ModelRunner.forward writes it to
    (model_runner.py:149-163): a prefill chunk writes positions
    [num_computed, num_computed + chunk), a decode row writes total_len - 1."""
    out = []
    for r in rows:
        if r["phase"] == "NEEDS_PREFILL":
            positions = range(r["num_computed_tokens"], r["num_computed_tokens"] + r["chunk"])
        else:
            positions = [r["total_len"] - 1]
        out.extend(flat_slot(r["block_table"], p) for p in positions)
    return out
