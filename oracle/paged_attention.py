"""Restatement of the reference's paged attention (TEST INFRASTRUCTURE ONLY).

Follows the reference kernel paged_flash_fwd_kernel
(serving_engine/paged_attention_kernel.py:16-122) and its launcher
(:125-160) per row, per query head, in float64 (or float32):

* row r has q_lens[r] queries starting at token q_starts[r]; query i sits at
  logical position q_pos_offsets[r] + i (:38-41, :103-106);
* keys are visited in 16-token blocks for blocks 0 .. ceil(k_len/16)-1 of the
  row's block table (:79-80); inside the last block, keys at or past k_len are
  zero-padded by the boundary-checked loads (:82-100), i.e. score 0, value 0;
* q-head h reads kv head h // (HQ / HKV) (:81);
* causal masking subtracts 1e6 from scores of keys after the query position
  (:104-109); exp(-1e6 + O(1)) is exactly 0 in fp32, so those keys are dropped
  here (a row always keeps key 0, so the -1e6 entries never set the max);
* O = sum_j exp(s_j - m) v_j / sum_j exp(s_j - m), LSE = m + log(l) (:111-119);
  a row with k_len = 0 yields O = 0/0 = NaN and LSE = -inf, as the reference
  does (its loop body never runs, :79, :118-119).

It equals the reference's eager oracle path (transformers
integrations/eager_paged.py:19-75 with the mask of model_runner.py:185-207)
for causal calls, which is what the model path always issues.
"""
from __future__ import annotations

import numpy as np

BLOCK_SIZE = 16


def _as_np(x, dtype=None):
    try:
        import torch

        if isinstance(x, torch.Tensor):
            x = x.detach().to("cpu")
            if x.dtype == torch.bfloat16 or x.dtype == torch.float16:
                x = x.float()
            x = x.numpy()
    except ImportError:  # pragma: no cover
        pass
    x = np.asarray(x)
    return x.astype(dtype) if dtype is not None else x


def gather_row_kv(k_cache, v_cache, block_table_row, k_len: int):
    """K/V of one row as [ceil16(k_len), HKV, D], zero past k_len (paged_attention_kernel.py:82-100)."""
    n_tiles = -(-int(k_len) // BLOCK_SIZE)
    hkv, d = k_cache.shape[2], k_cache.shape[3]
    k = np.zeros((n_tiles * BLOCK_SIZE, hkv, d), dtype=k_cache.dtype)
    v = np.zeros_like(k)
    for j in range(n_tiles):
        blk = int(block_table_row[j])
        n = min(BLOCK_SIZE, int(k_len) - j * BLOCK_SIZE)
        k[j * BLOCK_SIZE:j * BLOCK_SIZE + n] = k_cache[blk, :n]
        v[j * BLOCK_SIZE:j * BLOCK_SIZE + n] = v_cache[blk, :n]
    return k, v


def paged_attention(q, k_cache, v_cache, block_table, q_starts, q_lens, k_lens, q_pos_offsets,
                    scale: float, is_causal: bool = True, num_kv_heads: int | None = None,
                    dtype=np.float64, rows=None, heads=None):
    """Reference paged attention. Returns (o [total_q, HQ, D], lse [total_q, HQ]) in `dtype`.

    Inputs may be torch tensors or numpy arrays; bf16/fp16 inputs are upcast
    exactly. Entries of rows not listed in `rows` and of query heads not listed
    in `heads` (default: all) stay NaN.
    """
    q = _as_np(q, dtype)
    k_cache = _as_np(k_cache, dtype)
    v_cache = _as_np(v_cache, dtype)
    block_table = _as_np(block_table)
    q_starts, q_lens, k_lens, q_pos_offsets = (np.asarray(_as_np(a)).reshape(-1).astype(np.int64)
                                               for a in (q_starts, q_lens, k_lens, q_pos_offsets))
    total_q, hq, d = q.shape
    hkv = num_kv_heads if num_kv_heads is not None else k_cache.shape[2]
    group = hq // hkv
    o = np.full((total_q, hq, d), np.nan, dtype=dtype)
    lse = np.full((total_q, hq), np.nan, dtype=dtype)
    for r in (range(len(q_lens)) if rows is None else rows):
        nq, nk, qs, qp = int(q_lens[r]), int(k_lens[r]), int(q_starts[r]), int(q_pos_offsets[r])
        if nq <= 0:
            continue
        if nk <= 0:
            o[qs:qs + nq] = np.nan
            lse[qs:qs + nq] = -np.inf
            continue
        k, v = gather_row_kv(k_cache, v_cache, block_table[r], nk)
        n_keys = k.shape[0]
        allowed = np.ones((nq, n_keys), dtype=bool)
        if is_causal:
            allowed = (qp + np.arange(nq))[:, None] >= np.arange(n_keys)[None, :]
        for h in (range(hq) if heads is None else heads):
            kvh = h // group
            s = (q[qs:qs + nq, h] @ k[:, kvh].T) * dtype(scale)
            s = np.where(allowed, s, -np.inf)
            m = s.max(axis=1)
            p = np.exp(s - m[:, None])
            l = p.sum(axis=1)
            o[qs:qs + nq, h] = (p @ v[:, kvh]) / l[:, None]
            lse[qs:qs + nq, h] = m + np.log(l)
    return o, lse


def decode_rows(q, k_cache, v_cache, block_tables, k_lens, scale: float, rows, dtype=np.float64):
    """Decode (q_len = 1, q_pos = k_len - 1) rows only, with per-row host block tables.

    Gathers just the listed rows' blocks, so it is cheap on config-2 sized pools.
    Returns {row: (o [HQ, D], lse [HQ])}.
    """
    out = {}
    for r in rows:
        kl = int(k_lens[r])
        blocks = list(block_tables[r])
        n_tiles = -(-kl // BLOCK_SIZE)
        idx = blocks[:n_tiles]
        kc = _as_np(k_cache[idx], dtype)
        vc = _as_np(v_cache[idx], dtype)
        qr = _as_np(q[r:r + 1], dtype)
        o, lse = paged_attention(qr, kc, vc, np.arange(n_tiles)[None, :], [0], [1], [kl], [kl - 1], scale,
                                 True, dtype=dtype)
        out[r] = (o[0], lse[0])
    return out
