"""Cache shim and registered attention function for the Hugging Face model path.

``PagedKVCache`` is duck-typed like the reference's ``_PagedKVCache``
(serving_engine/model_runner.py:11-45): ``write`` scatters a layer's new K/V
into the pool (here one fused sm_100a launch instead of two ``index_copy_``),
``update`` keeps the reference's write-then-gather contract for the eager
oracle path, ``blocks`` returns the raw per-layer K/V views. ``copy_blocks``
is new: the batched copy-on-write copy for prefix-cache forks.

``b200_paged_attention_forward`` has the signature of the reference's
``triton_paged_attention_forward`` (model_runner.py:48-59) and is registered
under ``PAGED_B200_ATTN_IMPL = "paged|b200"`` in transformers'
ALL_ATTENTION_FUNCTIONS, so switching an engine to this backend is the one
string ``attn_implementation="paged|b200"``. It accepts the reference's own
``_PagedKVCache`` object as ``cache`` as well (it only uses ``blocks()`` and
``num_kv_heads``), so the reference ModelRunner runs unchanged.
"""
from __future__ import annotations

import torch

from . import ops
from .paged_attention import paged_flash_attention

PAGED_B200_ATTN_IMPL = "paged|b200"


class PagedKVCache:
    def __init__(self, kv_cache: torch.Tensor):
        self.kv_cache = kv_cache  # [num_layers, 2, num_blocks, block_size, num_kv_heads, head_dim]
        self.num_kv_heads = kv_cache.shape[-2]
        self.head_dim = kv_cache.shape[-1]

    def write(self, key_states, value_states, layer_idx, write_index):
        """key_states/value_states: [1, num_kv_heads, seq, head_dim] (any strides);
        write_index: int64 [seq] flat slots. One kernel launch for K and V."""
        k_cache, v_cache = self.blocks(layer_idx)
        ops.kv_append(key_states.transpose(1, 2).squeeze(0), value_states.transpose(1, 2).squeeze(0),
                      k_cache, v_cache, write_index)

    def update(self, key_states, value_states, layer_idx, read_index, write_index):
        """Eager oracle path: write, then gather a dense [n_read, num_kv_heads, head_dim] read."""
        self.write(key_states, value_states, layer_idx, write_index)
        k_cache = self.kv_cache[layer_idx, 0].view(-1, self.num_kv_heads, self.head_dim)
        v_cache = self.kv_cache[layer_idx, 1].view(-1, self.num_kv_heads, self.head_dim)
        return torch.index_select(k_cache, 0, read_index), torch.index_select(v_cache, 0, read_index)

    def blocks(self, layer_idx):
        return self.kv_cache[layer_idx, 0], self.kv_cache[layer_idx, 1]

    def copy_blocks(self, src, dst) -> None:
        """Copy blocks src[i] -> dst[i] in every layer and K/V plane (copy-on-write)."""
        ops.copy_blocks(self.kv_cache, src, dst)


def b200_paged_attention_forward(module, query, key, value, attention_mask, scaling, **kwargs):
    cache = kwargs["cache"]
    k_cache, v_cache = cache.blocks(module.layer_idx)
    ops.kv_append(key.transpose(1, 2).squeeze(0), value.transpose(1, 2).squeeze(0), k_cache, v_cache,
                  kwargs["write_index"])
    q = query.transpose(1, 2).squeeze(0)  # [1, heads, seq, dim] -> [seq, heads, dim]
    o, _ = paged_flash_attention(q, k_cache, v_cache, kwargs["paged_metadata"], num_q_heads=q.shape[1],
                                 num_kv_heads=cache.num_kv_heads, scale=scaling, is_causal=True)
    return o.unsqueeze(0), None  # [1, seq, heads, dim], the eager path's return layout


def register() -> str:
    """Register the attention function with transformers; returns its name."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    ALL_ATTENTION_FUNCTIONS.register(PAGED_B200_ATTN_IMPL, b200_paged_attention_forward)
    return PAGED_B200_ATTN_IMPL
