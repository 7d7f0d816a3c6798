"""B200 (sm_100a) paged-KV attention backend for the serving engine.

Public API mirrors the reference's hot-path modules:

* ``paged_flash_attention`` / ``build_paged_batch_metadata``
  (serving_engine/paged_attention_kernel.py)
* ``PagedKVCache`` (serving_engine/model_runner.py:_PagedKVCache) and the
  attention function registered as ``"paged|b200"``
* tensor ops ``kv_append``, ``copy_blocks``, ``paged_decode``, ``paged_prefill``
  over the C ABI in include/serving_engine_b200.h, and the decode-layer fusions
  ``rope_kv_append``, ``add_rmsnorm``, ``swiglu`` used by the tensor-parallel
  decoder.

Importing the package does not load the CUDA library; the first op does, and
raises if it has not been built (``python -m serving_engine_b200.build``).
"""
from .kv_cache import PAGED_B200_ATTN_IMPL, PagedKVCache, b200_paged_attention_forward, register
from .ops import (add_rmsnorm, check_device_errors, copy_blocks, kv_append, paged_decode, paged_prefill,
                  rope_kv_append, swiglu)
from .paged_attention import (PAGED_K_TILE_SIZE, PAGED_Q_TILE_SIZE, build_paged_batch_metadata,
                              metadata_from_lists, paged_flash_attention)

__all__ = [
    "PAGED_B200_ATTN_IMPL",
    "PAGED_K_TILE_SIZE",
    "PAGED_Q_TILE_SIZE",
    "PagedKVCache",
    "add_rmsnorm",
    "b200_paged_attention_forward",
    "build_paged_batch_metadata",
    "check_device_errors",
    "copy_blocks",
    "kv_append",
    "metadata_from_lists",
    "paged_decode",
    "paged_flash_attention",
    "paged_prefill",
    "register",
    "rope_kv_append",
    "swiglu",
]
