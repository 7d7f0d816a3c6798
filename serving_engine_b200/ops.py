"""Tensor-level wrappers over the C ABI (device memory and streams from torch).

Each op validates shapes, dtypes and devices on the host, without a device
sync, and enqueues its kernel on the current torch CUDA stream. Kernels report
out-of-range indices met at run time through a per-device int32 error word,
which ``check_device_errors()`` reads back (one sync) and raises on.
"""
from __future__ import annotations

import functools
import os
import threading

import torch

from . import _lib
from ._lib import SEB_BF16, SEB_F16, SEB_F32, check, lib

BLOCK_SIZE = 16  # serving_engine/block.py:7

_DTYPES = {torch.float32: SEB_F32, torch.float16: SEB_F16, torch.bfloat16: SEB_BF16}

_state = threading.local()
# Number of kernels each op enqueued so far (host-side count, read by bench.py).
LAUNCHES = [0]
_err_words: dict[int, torch.Tensor] = {}
_workspaces: dict[int, torch.Tensor] = {}
# Workspaces outgrown by a larger call stay allocated: a captured CUDA graph may
# still hold their address.
_retired_workspaces: list[torch.Tensor] = []

# SEB_DEBUG=1 checks the device error word after every op (one sync per op).
DEBUG = os.environ.get("SEB_DEBUG", "0") not in ("", "0")
# SEB_NVTX=1 wraps every op in an NVTX range named "seb.<op>" (for nsys / ncu
# --nvtx filtering); off, the ops are the plain functions.
NVTX = os.environ.get("SEB_NVTX", "0") not in ("", "0")


def _nvtx(fn):
    if not NVTX:
        return fn
    name = "seb." + fn.__name__

    @functools.wraps(fn)
    def wrapped(*args, **kwargs):
        torch.cuda.nvtx.range_push(name)
        try:
            return fn(*args, **kwargs)
        finally:
            torch.cuda.nvtx.range_pop()

    return wrapped


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16") from None


def _require_cuda(name: str, *tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise ValueError(f"{name}: tensors must be on a CUDA device, got {dev}")
    for t in tensors[1:]:
        if t.device != dev:
            raise ValueError(f"{name}: all tensors must be on {dev}, got {t.device}")
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def err_word(dev: torch.device) -> torch.Tensor:
    """The device's int32 error word (created zeroed on first use)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _err_words.get(idx)
    if w is None:
        # a normal tensor even when first touched under torch.inference_mode
        with torch.inference_mode(False):
            w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _err_words[idx] = w
    return w


def check_device_errors(dev: torch.device | None = None, reset: bool = True) -> None:
    """Sync, read the error word and raise RuntimeError naming its bits."""
    devs = [dev] if dev is not None else [torch.device("cuda", i) for i in list(_err_words)]
    for d in devs:
        w = err_word(d)
        bits = int(w.item())
        if reset:
            w.zero_()
        if bits:
            raise RuntimeError(f"serving_engine_b200 kernel error on {d}: " + ", ".join(_lib.decode_errbits(bits)))


def workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    """A per-device scratch buffer of at least nbytes, grown on demand to at
    least twice its size, so a run whose batches grow step by step reallocates
    a few times rather than at every step."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < nbytes:
        size = max(nbytes, 1 << 20)
        if ws is not None:
            _retired_workspaces.append(ws)
            size = max(size, 2 * ws.numel())
        with torch.inference_mode(False):
            ws = torch.empty(size, dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[idx] = ws
    return ws


def _after(dev: torch.device) -> None:
    if DEBUG:
        check_device_errors(dev)


# ------------------------------------------------------------------ kv append
@_nvtx
def kv_append(k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
              slot_mapping: torch.Tensor) -> None:
    """k_cache.view(-1, H, D)[slot_mapping] = k_new; same for V (one launch).

    k_new, v_new: [n_tokens, H, D] with unit stride on D (any token/head strides).
    k_cache, v_cache: [num_blocks, 16, H, D] contiguous. slot_mapping: int64 [n_tokens].
    Equivalent to the two index_copy_ of _PagedKVCache.write (model_runner.py:21-32).
    """
    dev = _require_cuda("kv_append", k_new, v_new, k_cache, v_cache, slot_mapping)
    if k_new.dim() != 3 or v_new.shape != k_new.shape:
        raise ValueError(f"kv_append: k_new/v_new must both be [n_tokens, H, D], got {tuple(k_new.shape)} "
                         f"and {tuple(v_new.shape)}")
    n, h, d = k_new.shape
    if k_cache.dim() != 4 or k_cache.shape[1] != BLOCK_SIZE or tuple(k_cache.shape[2:]) != (h, d):
        raise ValueError(f"kv_append: k_cache must be [num_blocks, {BLOCK_SIZE}, {h}, {d}], got {tuple(k_cache.shape)}")
    if v_cache.shape != k_cache.shape:
        raise ValueError("kv_append: k_cache and v_cache shapes differ")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("kv_append: KV caches must be contiguous")
    if not (k_new.dtype == v_new.dtype == k_cache.dtype == v_cache.dtype):
        raise ValueError("kv_append: dtype mismatch between new K/V and the cache")
    if k_new.stride(2) != 1 or v_new.stride(2) != 1:
        raise ValueError("kv_append: new K/V must have unit stride on head_dim")
    if slot_mapping.dtype != torch.int64 or slot_mapping.dim() != 1 or slot_mapping.numel() != n:
        raise ValueError(f"kv_append: slot_mapping must be int64 [{n}]")
    if not slot_mapping.is_contiguous():
        slot_mapping = slot_mapping.contiguous()
    st = lib().seb_kv_append(
        k_new.data_ptr(), k_new.stride(0), k_new.stride(1),
        v_new.data_ptr(), v_new.stride(0), v_new.stride(1),
        n, slot_mapping.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.shape[0], h, d, dtype_code(k_cache), err_word(dev).data_ptr(), _stream(dev))
    check("seb_kv_append", st)
    LAUNCHES[0] += 1
    _after(dev)


# ---------------------------------------------------------------- copy blocks
@_nvtx
def copy_blocks(kv_cache: torch.Tensor, src, dst) -> None:
    """kv_cache[:, :, dst] = kv_cache[:, :, src] for the engine pool
    [L, 2, num_blocks, 16, H, D] (model_runner.py:101-110), one launch.

    src/dst: sequences of block ids or int64 tensors. dst ids must be distinct
    and disjoint from src ids; host lists are validated here.
    """
    dev = _require_cuda("copy_blocks", kv_cache)
    if kv_cache.dim() != 6 or kv_cache.shape[1] != 2 or kv_cache.shape[3] != BLOCK_SIZE:
        raise ValueError(f"copy_blocks: pool must be [L, 2, num_blocks, {BLOCK_SIZE}, H, D], got {tuple(kv_cache.shape)}")
    if not kv_cache.is_contiguous():
        raise ValueError("copy_blocks: pool must be contiguous")
    nb = kv_cache.shape[2]
    src_t, dst_t = _block_ids(src, dev, "src"), _block_ids(dst, dev, "dst")
    if src_t.numel() != dst_t.numel():
        raise ValueError("copy_blocks: src and dst lengths differ")
    if not isinstance(src, torch.Tensor) and not isinstance(dst, torch.Tensor):
        s, d = list(src), list(dst)
        if len(set(d)) != len(d):
            raise ValueError("copy_blocks: duplicate dst block ids")
        if set(s) & set(d):
            raise ValueError("copy_blocks: a dst block is also a src block")
        bad = [b for b in s + d if not 0 <= int(b) < nb]
        if bad:
            raise ValueError(f"copy_blocks: block ids out of range [0, {nb}): {bad[:8]}")
    n = src_t.numel()
    if n == 0:
        return
    block_bytes = BLOCK_SIZE * kv_cache.shape[4] * kv_cache.shape[5] * kv_cache.element_size()
    layer_stride = kv_cache.stride(0) * kv_cache.element_size()
    st = lib().seb_copy_blocks(kv_cache.data_ptr(), kv_cache.shape[0], layer_stride, nb, block_bytes,
                               src_t.data_ptr(), dst_t.data_ptr(), n, err_word(dev).data_ptr(), _stream(dev))
    check("seb_copy_blocks", st)
    LAUNCHES[0] += 1
    _after(dev)


def _block_ids(x, dev: torch.device, name: str) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        if x.device != dev:
            raise ValueError(f"copy_blocks: {name} must be on {dev}")
        return x.to(torch.int64).contiguous()
    return torch.tensor(list(x), dtype=torch.int64).pin_memory().to(dev, non_blocking=True)


# --------------------------------------------------------------- paged decode
def decode_workspace_bytes(num_items: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                           max_blocks: int, blocks_per_split: int = 0) -> int:
    return int(lib().seb_paged_decode_workspace_size(num_items, num_q_heads, num_kv_heads, head_dim,
                                                     max_blocks, blocks_per_split))


@_nvtx
def decode_blocks_per_split(num_items: int, num_kv_heads: int, blocks_per_row: int, device=None,
                            num_sms: int | None = None) -> int:
    """Split length for seb_paged_decode when every row's length is known (here
    all rows hold `blocks_per_row` blocks). Splits are as long as possible (up
    to 64 blocks: fewer partials to merge) and balanced (the row divided into
    equal parts), with a split count whose warps (12 resident per SM) either
    fit in one wave, fill at least 40 % of their last wave, or make three waves
    or more: a short last wave leaves most SMs idle at the tail. Measured on the
    config-5 shards (256 rows of 256 blocks, head_dim 128): one kv head 97.0 us
    at 25 blocks (the former rule) against 91.1 at 64; two 174.3 at 32 against
    172.7 at 52; eight 649.0 against 638.3. The library's own default assumes
    rows fill half the block table. `num_sms` defaults to the device's SM count."""
    if num_sms is None:
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        num_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    slots = num_sms * 12
    blocks = max(blocks_per_row, 1)
    for splits in range(-(-blocks // 64), blocks + 1):
        bps = -(-blocks // splits)
        if bps < 8:
            break
        waves = num_items * num_kv_heads * splits / slots
        if waves <= 1.0 or waves >= 3.0 or waves - int(waves) >= 0.4:
            return bps
    return 8


def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                 q_starts: torch.Tensor, k_lens: torch.Tensor, q_pos_offsets: torch.Tensor,
                 num_q_heads: int, num_kv_heads: int, scale: float, is_causal: bool = True,
                 item_query: torch.Tensor | None = None, item_row: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
                 blocks_per_split: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Split-K paged attention for the listed query items (default: every token).

    q: [total_query, num_q_heads, D]; caches [num_blocks, 16, num_kv_heads, D];
    block_table int32 [rows, max_blocks]; q_starts/k_lens/q_pos_offsets int32 [rows].
    Returns (out like q, lse fp32 [total_query, num_q_heads]); rows of tokens that
    are not items are left untouched.

    The split-K scratch is one workspace per device, shared by every call on that
    device: calls on different streams must not run at the same time (calls in
    stream order, or inside one CUDA graph, are fine).
    """
    dev = _require_cuda("paged_decode", q, k_cache, v_cache, block_table, q_starts, k_lens, q_pos_offsets)
    if q.dim() != 3 or q.stride(2) != 1:
        raise ValueError(f"paged_decode: q must be [total_query, heads, head_dim] with unit inner stride, got {tuple(q.shape)}")
    total_q, hq, d = q.shape
    if hq != num_q_heads:
        raise ValueError(f"paged_decode: q has {hq} heads, num_q_heads={num_q_heads}")
    if num_kv_heads <= 0 or num_q_heads % num_kv_heads:
        raise ValueError(f"paged_decode: num_q_heads {num_q_heads} not a multiple of num_kv_heads {num_kv_heads}")
    if k_cache.dim() != 4 or k_cache.shape[1] != BLOCK_SIZE or tuple(k_cache.shape[2:]) != (num_kv_heads, d):
        raise ValueError(f"paged_decode: k_cache must be [num_blocks, {BLOCK_SIZE}, {num_kv_heads}, {d}], "
                         f"got {tuple(k_cache.shape)}")
    if v_cache.shape != k_cache.shape or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("paged_decode: k_cache and v_cache must be contiguous and of equal shape")
    if not (q.dtype == k_cache.dtype == v_cache.dtype):
        raise ValueError(f"paged_decode: dtype mismatch q {q.dtype}, cache {k_cache.dtype}")
    for name, t in (("block_table", block_table), ("q_starts", q_starts), ("k_lens", k_lens),
                    ("q_pos_offsets", q_pos_offsets)):
        if t.dtype != torch.int32:
            raise ValueError(f"paged_decode: {name} must be int32, got {t.dtype}")
    rows = q_starts.numel()
    if k_lens.numel() != rows or q_pos_offsets.numel() != rows:
        raise ValueError("paged_decode: q_starts, k_lens and q_pos_offsets lengths differ")
    if block_table.dim() != 2 or block_table.shape[0] != rows:
        raise ValueError(f"paged_decode: block_table must be [{rows}, max_blocks], got {tuple(block_table.shape)}")
    if block_table.stride(1) != 1:
        block_table = block_table.contiguous()
    q_starts, k_lens, q_pos_offsets = (t.contiguous() for t in (q_starts, k_lens, q_pos_offsets))
    max_blocks = block_table.shape[1]
    if item_query is not None:
        item_query = item_query.to(torch.int32).contiguous()
        num_items = item_query.numel()
    else:
        num_items = total_q
    if item_row is not None:
        item_row = item_row.to(torch.int32).contiguous()
        if item_row.numel() != num_items:
            raise ValueError("paged_decode: item_row length differs from the number of items")
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((total_q, num_q_heads), dtype=torch.float32, device=dev)
    if num_items == 0 or rows == 0 or max_blocks == 0:
        if num_items and rows:
            # no block table columns: every row has k_len 0 -> reference semantics O = NaN, LSE = -inf
            out.fill_(float("nan"))
            lse.fill_(float("-inf"))
        return out, lse
    ws_bytes = decode_workspace_bytes(num_items, num_q_heads, num_kv_heads, d, max_blocks, blocks_per_split)
    ws = workspace(dev, ws_bytes)
    st = lib().seb_paged_decode(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
        block_table.data_ptr(), block_table.stride(0), max_blocks,
        q_starts.data_ptr(), k_lens.data_ptr(), q_pos_offsets.data_ptr(),
        rows, total_q,
        item_query.data_ptr() if item_query is not None else None,
        item_row.data_ptr() if item_row is not None else None,
        num_items, num_q_heads, num_kv_heads, d, dtype_code(q),
        float(scale), 1 if is_causal else 0, int(blocks_per_split),
        out.data_ptr(), out.stride(0), out.stride(1),
        lse.data_ptr(), lse.stride(0),
        ws.data_ptr(), ws.numel(), err_word(dev).data_ptr(), _stream(dev))
    check("seb_paged_decode", st)
    LAUNCHES[0] += 1  # splits and their merge run in one launch
    _after(dev)
    return out, lse


# ------------------------------------------- whole batch, device-side routing
@_nvtx
def paged_attention_routed(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                           q_lens: torch.Tensor, k_lens: torch.Tensor, q_starts: torch.Tensor,
                           q_pos_offsets: torch.Tensor, num_q_heads: int, num_kv_heads: int, scale: float,
                           is_causal: bool = True, out: torch.Tensor | None = None,
                           lse: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Paged attention for a mixed batch described only by the reference's
    per-row device arrays (q_lens, k_lens, q_starts, q_pos_offsets, block_table:
    the dict of build_paged_batch_metadata). The rows are split into decode items
    and tcgen05 prefill units on the device (seb_paged_attention); the host reads
    nothing back."""
    dev = _require_cuda("paged_attention_routed", q, k_cache, v_cache, block_table, q_lens, k_lens, q_starts,
                        q_pos_offsets)
    if q.dim() != 3 or q.stride(2) != 1 or q.shape[1] != num_q_heads:
        raise ValueError(f"paged_attention_routed: q must be [total_query, {num_q_heads}, head_dim] with unit inner "
                         f"stride, got {tuple(q.shape)}")
    total_q, hq, d = q.shape
    if num_kv_heads <= 0 or num_q_heads % num_kv_heads:
        raise ValueError(f"paged_attention_routed: num_q_heads {num_q_heads} not a multiple of {num_kv_heads}")
    if k_cache.dim() != 4 or k_cache.shape[1] != BLOCK_SIZE or tuple(k_cache.shape[2:]) != (num_kv_heads, d):
        raise ValueError(f"paged_attention_routed: k_cache must be [num_blocks, {BLOCK_SIZE}, {num_kv_heads}, {d}]")
    if v_cache.shape != k_cache.shape or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("paged_attention_routed: k_cache and v_cache must be contiguous and of equal shape")
    if not (q.dtype == k_cache.dtype == v_cache.dtype):
        raise ValueError("paged_attention_routed: dtype mismatch")
    for name, t in (("block_table", block_table), ("q_lens", q_lens), ("k_lens", k_lens), ("q_starts", q_starts),
                    ("q_pos_offsets", q_pos_offsets)):
        if t.dtype != torch.int32:
            raise ValueError(f"paged_attention_routed: {name} must be int32")
    rows = q_lens.numel()
    if not (k_lens.numel() == q_starts.numel() == q_pos_offsets.numel() == rows):
        raise ValueError("paged_attention_routed: per-row arrays differ in length")
    if block_table.dim() != 2 or block_table.shape[0] != rows:
        raise ValueError(f"paged_attention_routed: block_table must be [{rows}, max_blocks]")
    if block_table.stride(1) != 1:
        block_table = block_table.contiguous()
    q_lens, k_lens, q_starts, q_pos_offsets = (t.contiguous() for t in (q_lens, k_lens, q_starts, q_pos_offsets))
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((total_q, num_q_heads), dtype=torch.float32, device=dev)
    max_blocks = block_table.shape[1]
    if rows == 0 or total_q == 0:
        return out, lse
    if max_blocks == 0:
        out.fill_(float("nan"))  # every row has k_len 0: O = NaN, LSE = -inf (reference semantics)
        lse.fill_(float("-inf"))
        return out, lse
    nbytes = int(lib().seb_paged_attention_workspace_size(rows, total_q, num_q_heads, num_kv_heads, d, max_blocks))
    ws = workspace(dev, nbytes)
    st = lib().seb_paged_attention(
        q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
        block_table.data_ptr(), block_table.stride(0), max_blocks, q_lens.data_ptr(), k_lens.data_ptr(),
        q_starts.data_ptr(), q_pos_offsets.data_ptr(), rows, total_q, num_q_heads, num_kv_heads, d, dtype_code(q),
        float(scale), 1 if is_causal else 0, out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
        lse.stride(0), ws.data_ptr(), ws.numel(), err_word(dev).data_ptr(), _stream(dev))
    check("seb_paged_attention", st)
    LAUNCHES[0] += 3 if (total_q > rows and prefill_supported(q, num_q_heads, num_kv_heads)) else 1
    _after(dev)
    return out, lse


# -------------------------------------------------------------- paged prefill
PREFILL_HEAD_DIMS = (64, 128)
PREFILL_GROUPS = (1, 2, 4, 8, 16)


def prefill_supported(q: torch.Tensor, num_q_heads: int, num_kv_heads: int) -> bool:
    """Whether the tcgen05 chunked-prefill kernel covers this dtype and shape."""
    if q.dtype not in (torch.bfloat16, torch.float16) or q.dim() != 3:
        return False
    if num_kv_heads <= 0 or num_q_heads % num_kv_heads:
        return False
    d = q.shape[2]
    return (d in PREFILL_HEAD_DIMS and num_q_heads // num_kv_heads in PREFILL_GROUPS and q.stride(2) == 1
            and q.stride(0) % 8 == 0 and q.stride(1) % 8 == 0 and q.data_ptr() % 16 == 0
            and q.stride(1) >= d and q.stride(0) >= q.stride(1) * num_q_heads)


@_nvtx
def paged_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                  q_starts: torch.Tensor, q_lens: torch.Tensor, k_lens: torch.Tensor, q_pos_offsets: torch.Tensor,
                  num_q_heads: int, num_kv_heads: int, scale: float, is_causal: bool = True, *,
                  max_q_len: int, rows: torch.Tensor | None = None, num_prefill_rows: int | None = None,
                  out: torch.Tensor | None = None, lse: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Chunked-prefill paged attention on tcgen05 tensor cores for the listed rows
    (default: every row). max_q_len: host-known bound of those rows' q_lens."""
    dev = _require_cuda("paged_prefill", q, k_cache, v_cache, block_table, q_starts, q_lens, k_lens, q_pos_offsets)
    if not prefill_supported(q, num_q_heads, num_kv_heads):
        raise ValueError("paged_prefill: needs bf16/fp16 q [total_query, heads, 64|128] with 16-byte aligned rows "
                         "and a GQA group of 1, 2, 4, 8 or 16")
    total_q, hq, d = q.shape
    if hq != num_q_heads:
        raise ValueError(f"paged_prefill: q has {hq} heads, num_q_heads={num_q_heads}")
    if k_cache.dim() != 4 or k_cache.shape[1] != BLOCK_SIZE or tuple(k_cache.shape[2:]) != (num_kv_heads, d):
        raise ValueError(f"paged_prefill: k_cache must be [num_blocks, {BLOCK_SIZE}, {num_kv_heads}, {d}]")
    if v_cache.shape != k_cache.shape or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("paged_prefill: k_cache and v_cache must be contiguous and of equal shape")
    if not (q.dtype == k_cache.dtype == v_cache.dtype):
        raise ValueError("paged_prefill: dtype mismatch")
    for name, t in (("block_table", block_table), ("q_starts", q_starts), ("q_lens", q_lens), ("k_lens", k_lens),
                    ("q_pos_offsets", q_pos_offsets)):
        if t.dtype != torch.int32:
            raise ValueError(f"paged_prefill: {name} must be int32")
    n_rows = q_starts.numel()
    if block_table.dim() != 2 or block_table.shape[0] != n_rows or block_table.stride(1) != 1:
        raise ValueError("paged_prefill: block_table must be [rows, max_blocks] with unit column stride")
    if rows is not None:
        rows = rows.to(torch.int32).contiguous()
        num_prefill_rows = rows.numel() if num_prefill_rows is None else num_prefill_rows
    elif num_prefill_rows is None:
        num_prefill_rows = n_rows
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((total_q, num_q_heads), dtype=torch.float32, device=dev)
    if out.stride(2) != 1 or out.stride(0) % 8 or out.stride(1) % 8 or out.data_ptr() % 16:
        raise ValueError("paged_prefill: out rows must be 16-byte aligned")
    if num_prefill_rows == 0 or max_q_len == 0 or block_table.shape[1] == 0:
        return out, lse
    q_starts, q_lens, k_lens, q_pos_offsets = (t.contiguous() for t in (q_starts, q_lens, k_lens, q_pos_offsets))
    st = lib().seb_paged_prefill(
        q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
        block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
        q_starts.data_ptr(), q_lens.data_ptr(), k_lens.data_ptr(), q_pos_offsets.data_ptr(), n_rows, total_q,
        rows.data_ptr() if rows is not None else None, int(num_prefill_rows), int(max_q_len),
        num_q_heads, num_kv_heads, d, dtype_code(q), float(scale), 1 if is_causal else 0,
        out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0),
        err_word(dev).data_ptr(), _stream(dev))
    check("seb_paged_prefill", st)
    LAUNCHES[0] += 1
    _after(dev)
    return out, lse


# ------------------------------------------------------ decode-layer fusions
def _half_dtype(name: str, *tensors: torch.Tensor) -> int:
    dt = tensors[0].dtype
    if dt not in (torch.bfloat16, torch.float16) or any(t.dtype != dt for t in tensors):
        raise ValueError(f"{name}: all tensors must share one dtype, bf16 or fp16")
    return dtype_code(tensors[0])


@_nvtx
def rope_kv_append(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, slot_mapping: torch.Tensor,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """Rotary embedding fused with the KV write: returns q rotated
    [n_tokens, num_q_heads, head_dim] and writes rotated K and V of token t to
    pool slot slot_mapping[t] (one launch).

    qkv: [n_tokens, (num_q_heads + 2 * num_kv_heads) * head_dim] (q heads, then
    k heads, then v heads); cos/sin: [n_tokens, head_dim] (any leading views that
    flatten to that, unit stride on head_dim); k_cache/v_cache: [num_blocks, 16,
    num_kv_heads, head_dim] contiguous. Bit-identical to
    ``x * cos + rotate_half(x) * sin`` in the element type followed by
    kv_append.
    """
    dev = _require_cuda("rope_kv_append", qkv, cos, sin, slot_mapping, k_cache, v_cache)
    dt = _half_dtype("rope_kv_append", qkv, cos, sin, k_cache, v_cache)
    if qkv.dim() != 2 or qkv.stride(1) != 1:
        raise ValueError("rope_kv_append: qkv must be [n_tokens, width] with unit column stride")
    n = qkv.shape[0]
    if k_cache.dim() != 4 or k_cache.shape[1] != BLOCK_SIZE or k_cache.shape[2] != num_kv_heads:
        raise ValueError(f"rope_kv_append: k_cache must be [num_blocks, {BLOCK_SIZE}, {num_kv_heads}, head_dim]")
    d = k_cache.shape[3]
    if qkv.shape[1] != (num_q_heads + 2 * num_kv_heads) * d:
        raise ValueError(f"rope_kv_append: qkv width {qkv.shape[1]} != ({num_q_heads} + 2 x {num_kv_heads}) x {d}")
    if v_cache.shape != k_cache.shape or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("rope_kv_append: k_cache and v_cache must be contiguous and of equal shape")
    cos2, sin2 = cos.reshape(-1, cos.shape[-1]), sin.reshape(-1, sin.shape[-1])
    if cos2.shape != (n, d) or sin2.shape != (n, d) or cos2.stride() != sin2.stride() or cos2.stride(1) != 1:
        raise ValueError(f"rope_kv_append: cos and sin must be [n_tokens={n}, head_dim={d}] with equal strides")
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() != n:
        raise ValueError(f"rope_kv_append: slot_mapping must be int64 [{n}]")
    slot_mapping = slot_mapping.contiguous()
    if out is None:
        out = torch.empty(n, num_q_heads, d, dtype=qkv.dtype, device=dev)
    elif out.shape != (n, num_q_heads, d) or out.stride(2) != 1 or out.stride(1) != d:
        raise ValueError("rope_kv_append: out must be [n_tokens, num_q_heads, head_dim] with contiguous heads")
    st = lib().seb_rope_kv_append(qkv.data_ptr(), qkv.stride(0), n, num_q_heads, num_kv_heads, d,
                                  cos2.data_ptr(), sin2.data_ptr(), cos2.stride(0), slot_mapping.data_ptr(),
                                  out.data_ptr(), out.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                                  k_cache.shape[0], dt, err_word(dev).data_ptr(), _stream(dev))
    check("seb_rope_kv_append", st)
    LAUNCHES[0] += 1
    _after(dev)
    return out


@_nvtx
def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor, eps: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """x += residual (in place, when given), then RMSNorm(x) * weight, one launch.

    x, residual, out: [n_rows, hidden] with unit column stride; weight: [hidden].
    """
    ts = (x, weight) if residual is None else (x, residual, weight)
    dev = _require_cuda("add_rmsnorm", *ts)
    dt = _half_dtype("add_rmsnorm", *ts)
    if x.dim() != 2 or x.stride(1) != 1 or weight.shape != (x.shape[1],) or not weight.is_contiguous():
        raise ValueError("add_rmsnorm: x must be [n_rows, hidden] (unit column stride), weight [hidden]")
    if residual is not None and (residual.shape != x.shape or residual.stride(1) != 1):
        raise ValueError("add_rmsnorm: residual must match x")
    if out is None:
        out = torch.empty_like(x)
    elif out.shape != x.shape or out.stride(1) != 1 or out.dtype != x.dtype:
        raise ValueError("add_rmsnorm: out must match x")
    st = lib().seb_add_rmsnorm(x.data_ptr(), x.stride(0), 0 if residual is None else residual.data_ptr(),
                               0 if residual is None else residual.stride(0), weight.data_ptr(), out.data_ptr(),
                               out.stride(0), x.shape[0], x.shape[1], float(eps), dt, _stream(dev))
    check("seb_add_rmsnorm", st)
    LAUNCHES[0] += 1
    _after(dev)
    return out


@_nvtx
def swiglu(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate) * up for gate_up = [gate | up] of shape [n_rows, 2 * ffn], one launch."""
    dev = _require_cuda("swiglu", gate_up)
    dt = _half_dtype("swiglu", gate_up)
    if gate_up.dim() != 2 or gate_up.stride(1) != 1 or gate_up.shape[1] % 2:
        raise ValueError("swiglu: gate_up must be [n_rows, 2 * ffn] with unit column stride")
    n, f = gate_up.shape[0], gate_up.shape[1] // 2
    if out is None:
        out = torch.empty(n, f, dtype=gate_up.dtype, device=dev)
    elif out.shape != (n, f) or out.stride(1) != 1 or out.dtype != gate_up.dtype:
        raise ValueError("swiglu: out must be [n_rows, ffn]")
    st = lib().seb_swiglu(gate_up.data_ptr(), gate_up.stride(0), out.data_ptr(), out.stride(0), n, f, dt, _stream(dev))
    check("seb_swiglu", st)
    LAUNCHES[0] += 1
    _after(dev)
    return out


# ------------------------------------------------------------- failure self-test
def selftest_bounded_wait(polls: int = 4096, device=None) -> None:
    """Launch the bounded-wait self-test: it waits on an mbarrier nothing arrives
    on, gives up after `polls` polls and sets SEB_ERRBIT_TIMEOUT in the device's
    error word (read it with check_device_errors)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    st = lib().seb_selftest_bounded_wait(int(polls), err_word(dev).data_ptr(), _stream(dev))
    check("seb_selftest_bounded_wait", st)
