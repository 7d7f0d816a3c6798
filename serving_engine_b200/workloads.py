"""Seeded synthetic inputs with the shapes of the reference's configurations.

The reference measures on synthetic data only (serving_engine/workload.py,
scripts/benchmark_load.py:29-31 use random token ids); these generators build
the paged-attention inputs of the configurations this backend is measured on:

* config 1 -- fp32 decode, 8 sequences, k_len ~ U[1, 512], 12 q heads = 12 kv
  heads, head_dim 64, pool 512 blocks, each table a seeded permutation slice.
* config 2 -- bf16 GQA decode (Llama-3-8B attention shape), 64 sequences,
  k_len ~ U[1024, 8192], 32 q heads, 8 kv heads, head_dim 128, pool of
  ceil(1.25 * sum(k_len) / 16) blocks with shuffled block tables.
* config 3 -- bf16 chunked prefill with prefix caching: 16 sequences share a
  2048-token prefix (the same physical blocks) and each appends a distinct
  512-token causal chunk into fresh blocks.

All host-side randomness comes from ``torch.Generator().manual_seed(seed)``
(CPU), so the same seed gives bit-identical inputs on every machine with this
torch build. Large pools can be filled on the GPU instead (``fill="cuda"``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

BLOCK_SIZE = 16


@dataclass
class PagedBatch:
    """One paged-attention call: queries, pool and the reference's metadata."""

    q: torch.Tensor                 # [total_query, HQ, D]
    k_cache: torch.Tensor           # [num_blocks, 16, HKV, D]
    v_cache: torch.Tensor
    block_tables: list[list[int]]   # per row, physical block ids
    q_lens: list[int]
    k_lens: list[int]
    q_pos_offsets: list[int]
    num_q_heads: int
    num_kv_heads: int
    scale: float
    extra: dict = field(default_factory=dict)

    @property
    def q_starts(self) -> list[int]:
        out, s = [], 0
        for n in self.q_lens:
            out.append(s)
            s += n
        return out

    @property
    def head_dim(self) -> int:
        return self.q.shape[-1]

    def metadata(self, device) -> dict:
        """The dict build_paged_batch_metadata returns (paged_attention_kernel.py:193-200)."""
        max_blocks = max((len(bt) for bt in self.block_tables), default=0)
        padded = [bt + [0] * (max_blocks - len(bt)) for bt in self.block_tables]
        i32 = dict(dtype=torch.int32, device=device)
        return {
            "q_lens": torch.tensor(self.q_lens, **i32),
            "k_lens": torch.tensor(self.k_lens, **i32),
            "q_starts": torch.tensor(self.q_starts, **i32),
            "q_pos_offsets": torch.tensor(self.q_pos_offsets, **i32),
            "block_table": torch.tensor(padded, **i32).reshape(len(self.block_tables), max_blocks),
            "block_table_row_stride": max_blocks,
            "total_query": sum(self.q_lens),
        }

    def kv_bytes(self) -> int:
        """Algorithmic KV bytes of the call: sum k_len * HKV * D * 2 (K, V) * elem."""
        return sum(self.k_lens) * self.num_kv_heads * self.head_dim * 2 * self.k_cache.element_size()


def _fill(shape, dtype, gen: torch.Generator, fill: str, seed: int) -> torch.Tensor:
    if fill == "cpu":
        return torch.randn(shape, generator=gen, dtype=torch.float32).to(dtype)
    g = torch.Generator(device=fill).manual_seed(seed)
    out = torch.empty(shape, dtype=dtype, device=fill)
    # fill in chunks so the fp32 staging stays small
    flat = out.view(-1)
    step = 1 << 26
    for i in range(0, flat.numel(), step):
        n = min(step, flat.numel() - i)
        flat[i:i + n] = torch.randn(n, generator=g, device=fill, dtype=torch.float32).to(dtype)
    return out


def decode_k_lens(batch: int, k_min: int, k_max: int, seed: int) -> list[int]:
    """The k_len draw of decode_batch(batch, k_min, k_max, ..., seed): U[k_min, k_max]."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(k_min, k_max + 1, (batch,), generator=gen).tolist()


def decode_batch(batch: int, k_min: int, k_max: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, seed: int, num_blocks: int | None = None, pool_factor: float = 1.25,
                 fill: str = "cpu", k_lens: list[int] | None = None) -> PagedBatch:
    """Decode batch: one query per sequence at its last position, k_len ~ U[k_min, k_max]
    (or the given per-sequence k_lens; tables, q and the pool still come from `seed`)."""
    gen = torch.Generator().manual_seed(seed)
    drawn = torch.randint(k_min, k_max + 1, (batch,), generator=gen).tolist()
    if k_lens is None:
        k_lens = drawn
    elif len(k_lens) != batch:
        raise ValueError(f"k_lens has {len(k_lens)} entries for a batch of {batch}")
    need = [math.ceil(k / BLOCK_SIZE) for k in k_lens]
    if num_blocks is None:
        num_blocks = max(math.ceil(pool_factor * sum(k_lens) / BLOCK_SIZE), sum(need))
    if sum(need) > num_blocks:
        raise ValueError(f"pool of {num_blocks} blocks cannot hold {sum(need)} blocks")
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    tables, pos = [], 0
    for n in need:
        tables.append(perm[pos:pos + n])
        pos += n
    q = _fill((batch, num_q_heads, head_dim), dtype, gen, "cpu", seed)
    cache_shape = (num_blocks, BLOCK_SIZE, num_kv_heads, head_dim)
    k_cache = _fill(cache_shape, dtype, gen, fill, seed + 1)
    v_cache = _fill(cache_shape, dtype, gen, fill, seed + 2)
    return PagedBatch(q=q, k_cache=k_cache, v_cache=v_cache, block_tables=tables, q_lens=[1] * batch,
                      k_lens=k_lens, q_pos_offsets=[k - 1 for k in k_lens], num_q_heads=num_q_heads,
                      num_kv_heads=num_kv_heads, scale=1.0 / math.sqrt(head_dim))


def config1(seed: int = 0) -> PagedBatch:
    return decode_batch(8, 1, 512, 12, 12, 64, torch.float32, seed, num_blocks=512)


def config2(seed: int = 0, batch: int = 64, fill: str = "cpu") -> PagedBatch:
    return decode_batch(batch, 1024, 8192, 32, 8, 128, torch.bfloat16, seed, fill=fill)


def prefix_prefill_batch(num_seqs: int, prefix_len: int, chunk_len: int, num_q_heads: int, num_kv_heads: int,
                         head_dim: int, dtype: torch.dtype, seed: int, fill: str = "cpu") -> PagedBatch:
    """Config-3 shape: every row shares the prefix blocks, then prefills its own chunk.

    The prefix's last block is shared too when prefix_len % 16 != 0; the caller
    then copies it (copy-on-write) into each row's first private block, which
    ``extra["cow_src"]`` / ``extra["cow_dst"]`` name. Rows' metadata describe the
    chunk prefill: q_len = chunk_len, q_pos_offset = prefix_len,
    k_len = prefix_len + chunk_len. ``extra["new_k"]``/``extra["new_v"]`` hold the
    chunk's K/V ([total_query, HKV, D]) and ``extra["slot_mapping"]`` their slots.
    """
    gen = torch.Generator().manual_seed(seed)
    full_prefix = prefix_len // BLOCK_SIZE
    partial = prefix_len % BLOCK_SIZE
    n_prefix_blocks = full_prefix + (1 if partial else 0)
    own = math.ceil((prefix_len + chunk_len) / BLOCK_SIZE) - full_prefix
    num_blocks = n_prefix_blocks + num_seqs * own + 8
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    prefix_blocks = perm[:n_prefix_blocks]
    pos = n_prefix_blocks
    tables, cow_src, cow_dst = [], [], []
    for _ in range(num_seqs):
        mine = perm[pos:pos + own]
        pos += own
        tables.append(prefix_blocks[:full_prefix] + mine)
        if partial:
            cow_src.append(prefix_blocks[full_prefix])
            cow_dst.append(mine[0])
    total_q = num_seqs * chunk_len
    q = _fill((total_q, num_q_heads, head_dim), dtype, gen, "cpu", seed)
    new_k = _fill((total_q, num_kv_heads, head_dim), dtype, gen, "cpu", seed)
    new_v = _fill((total_q, num_kv_heads, head_dim), dtype, gen, "cpu", seed)
    cache_shape = (num_blocks, BLOCK_SIZE, num_kv_heads, head_dim)
    k_cache = _fill(cache_shape, dtype, gen, fill, seed + 1)
    v_cache = _fill(cache_shape, dtype, gen, fill, seed + 2)
    slots = []
    for bt in tables:
        for p in range(prefix_len, prefix_len + chunk_len):
            slots.append(bt[p // BLOCK_SIZE] * BLOCK_SIZE + p % BLOCK_SIZE)
    return PagedBatch(
        q=q, k_cache=k_cache, v_cache=v_cache, block_tables=tables, q_lens=[chunk_len] * num_seqs,
        k_lens=[prefix_len + chunk_len] * num_seqs, q_pos_offsets=[prefix_len] * num_seqs,
        num_q_heads=num_q_heads, num_kv_heads=num_kv_heads, scale=1.0 / math.sqrt(head_dim),
        extra={"new_k": new_k, "new_v": new_v, "slot_mapping": torch.tensor(slots, dtype=torch.int64),
               "cow_src": cow_src, "cow_dst": cow_dst, "prefix_blocks": prefix_blocks})


def config3(seed: int = 0, prefix_len: int = 2048, fill: str = "cpu") -> PagedBatch:
    return prefix_prefill_batch(16, prefix_len, 512, 32, 8, 128, torch.bfloat16, seed, fill=fill)
