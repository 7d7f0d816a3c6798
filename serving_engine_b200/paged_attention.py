"""Drop-in for serving_engine/paged_attention_kernel.py on B200.

Same public names, signatures and return values as the reference module:

* ``paged_flash_attention(q, k_cache, v_cache, metadata, num_q_heads,
  num_kv_heads, scale, is_causal=True) -> (o, l)``
  (paged_attention_kernel.py:125-160), and
* ``build_paged_batch_metadata(scheduler_output, device="cuda") -> dict``
  (paged_attention_kernel.py:163-200),

but the attention runs in the sm_100a library (no Triton, no CPU path). The
metadata dict keeps every key the reference returns and adds a few host-known
values (``max_q_len``, per-token rows, ...) so the launcher never has to read a
device tensor back: the reference's per-layer ``q_lens.max().item()`` sync
(paged_attention_kernel.py:133) is gone. A metadata dict built elsewhere (e.g.
by the reference's own builder) is accepted too; rows are then located on the
device by binary search over q_starts.
"""
from __future__ import annotations

import itertools

import numpy as np
import torch

from . import ops

PAGED_K_TILE_SIZE = ops.BLOCK_SIZE  # one physical block per key tile (paged_attention_kernel.py:12)
PAGED_Q_TILE_SIZE = 16


def _is_prefill(req) -> bool:
    # RequestPhase.NEEDS_PREFILL of serving_engine/request.py:9-18, compared by
    # name so this module does not import the engine package.
    phase = req.phase
    return getattr(phase, "name", phase) == "NEEDS_PREFILL"


def build_paged_batch_metadata(scheduler_output, device="cuda") -> dict:
    """Per-step metadata, reused by every layer of the step.

    Row semantics follow paged_attention_kernel.py:171-187: a prefill row gets
    q_len = its chunk, k_len = num_computed_tokens + chunk, q_pos_offset =
    num_computed_tokens; a decode row gets q_len = 1, k_len = total_len,
    q_pos_offset = total_len - 1. Block tables are zero-padded to the widest row.
    All int32 arrays travel in ONE host-to-device copy from pinned memory.
    """
    q_lens, k_lens, q_starts, q_pos_offsets, tables = [], [], [], [], []
    start = 0
    for req in scheduler_output.scheduled_requests:
        if _is_prefill(req):
            nq = scheduler_output.prefill_chunk_sizes[req.request_id]
            nk = req.num_computed_tokens + nq
            qp = req.num_computed_tokens
        else:
            nq = 1
            nk = req.total_len
            qp = req.total_len - 1
        q_lens.append(nq)
        k_lens.append(nk)
        q_starts.append(start)
        q_pos_offsets.append(qp)
        tables.append(req.block_table)
        start += nq
    return metadata_from_lists(q_lens, k_lens, q_starts, q_pos_offsets, tables, device)


class PackedMetadata:
    """Host side of one step's metadata: every int32 array in one buffer.

    Layout: q_lens[R] | k_lens[R] | q_starts[R] | q_pos_offsets[R] |
    block_table[R, W] | item_row[total_query] | decode tokens[Nd] |
    decode rows[Nd] | prefill rows[Np], where decode rows are those with
    q_len == 1 and prefill rows those with q_len > 1. ``upload`` issues ONE
    host-to-device copy (pinned) and returns the metadata dict.
    """

    def __init__(self, q_lens, k_lens, q_starts, q_pos_offsets, tables):
        rows = len(q_lens)
        q_lens_np = np.asarray(q_lens, dtype=np.int32).reshape(rows)
        lens = np.fromiter((len(t) for t in tables), dtype=np.int64, count=rows)
        width = int(lens.max()) if rows else 0
        total_query = int(q_lens_np.sum())
        o_bt = 4 * rows
        o_items = o_bt + rows * width
        n_dec = int((q_lens_np == 1).sum())
        n_pre = int((q_lens_np > 1).sum())
        packed = torch.zeros(o_items + total_query + 2 * n_dec + n_pre, dtype=torch.int32)
        a = packed.numpy()
        a[0:rows] = q_lens_np
        a[rows:2 * rows] = k_lens
        a[2 * rows:3 * rows] = q_starts
        a[3 * rows:4 * rows] = q_pos_offsets
        n_ids = int(lens.sum())
        if n_ids:
            flat = np.fromiter(itertools.chain.from_iterable(tables), dtype=np.int32, count=n_ids)
            # destination of id k of row r: o_bt + r * width + k
            starts = np.repeat(np.arange(rows, dtype=np.int64) * width - np.concatenate(([0], np.cumsum(lens)[:-1])),
                               lens)
            a[o_bt + starts + np.arange(n_ids)] = flat
            self.max_block_id = int(flat.max())
        else:
            self.max_block_id = -1
        a[o_items:o_items + total_query] = np.repeat(np.arange(rows, dtype=np.int32), q_lens_np)
        # decode items (rows with q_len == 1: token, row) and prefill rows (q_len > 1).
        # Decode items go longest context first: the kernel's work is dispatched in
        # item order, so the short items fill the tail.
        dec_rows = np.nonzero(q_lens_np == 1)[0].astype(np.int32)
        dec_rows = dec_rows[np.argsort(-np.asarray(k_lens, dtype=np.int64).reshape(rows)[dec_rows], kind="stable")]
        pre_rows = np.nonzero(q_lens_np > 1)[0].astype(np.int32)
        starts_np = a[2 * rows:3 * rows]
        o_dec = o_items + total_query
        a[o_dec:o_dec + len(dec_rows)] = starts_np[dec_rows]
        a[o_dec + len(dec_rows):o_dec + 2 * len(dec_rows)] = dec_rows
        a[o_dec + 2 * len(dec_rows):] = pre_rows
        self.num_decode = len(dec_rows)
        self.num_prefill = len(pre_rows)
        self.max_prefill_q_len = int(q_lens_np[pre_rows].max()) if len(pre_rows) else 0
        self.host = packed
        self.rows, self.width, self.total_query = rows, width, total_query
        self.max_q_len = int(q_lens_np.max()) if rows else 0
        self.max_k_len = int(np.max(k_lens)) if rows else 0

    def pin(self) -> "PackedMetadata":
        if not self.host.is_pinned():
            self.host = self.host.pin_memory()
        return self

    @property
    def nbytes(self) -> int:
        return self.host.numel() * 4

    def upload(self, device="cuda", staging: torch.Tensor | None = None) -> dict:
        """Copy the buffer to `device` (one host-to-device copy) and return the
        metadata dict over it. `staging`: a pinned int32 host buffer of at least
        the packed size to copy through (the caller keeps it unwritten until the
        copy has run); otherwise the buffer is pinned for the copy."""
        dev = torch.device(device)
        if dev.type == "cuda" and staging is not None:
            st = staging[:self.host.numel()]
            st.copy_(self.host)
            buf = st.to(dev, non_blocking=True)
        elif dev.type == "cuda":
            buf = (self.host if self.host.is_pinned() else self.host.pin_memory()).to(dev, non_blocking=True)
        else:
            buf = self.host.clone()
        rows, width = self.rows, self.width
        o = 4 * rows
        o_dec = o + rows * width + self.total_query
        nd = self.num_decode
        return {
            "q_lens": buf[0:rows],
            "k_lens": buf[rows:2 * rows],
            "q_starts": buf[2 * rows:3 * rows],
            "q_pos_offsets": buf[3 * rows:4 * rows],
            "block_table": buf[o:o + rows * width].view(rows, width),
            "block_table_row_stride": width,
            "total_query": self.total_query,
            # host-known extras (not in the reference's dict)
            "max_q_len": self.max_q_len,
            "item_row": buf[o + rows * width:o + rows * width + self.total_query],
            "max_block_id": self.max_block_id,
            "max_k_len": self.max_k_len,
            "decode_tokens": buf[o_dec:o_dec + nd],
            "decode_rows": buf[o_dec + nd:o_dec + 2 * nd],
            "prefill_rows": buf[o_dec + 2 * nd:o_dec + 2 * nd + self.num_prefill],
            "max_prefill_q_len": self.max_prefill_q_len,
        }


class DecodeMetadataBuffer:
    """Fixed-shape step metadata for a decode-only batch of `rows` rows and a
    block-table width `width`, resident in one device buffer whose address never
    changes (what a captured CUDA graph reads). Layout as PackedMetadata with
    q_len = 1 for every row: q_lens | k_lens | q_starts | q_pos_offsets |
    block_table | item_row | decode tokens | decode rows (no prefill rows); each
    update lists the decode items longest context first."""

    def __init__(self, rows: int, width: int, device):
        self.rows, self.width = rows, width
        n = 4 * rows + rows * width + 3 * rows
        host = torch.zeros(n, dtype=torch.int32)
        a = host.numpy()
        ar = np.arange(rows, dtype=np.int32)
        a[0:rows] = 1
        a[2 * rows:3 * rows] = ar
        o = 4 * rows + rows * width
        a[o:o + rows] = ar          # item_row
        a[o + rows:o + 2 * rows] = ar  # decode tokens
        a[o + 2 * rows:o + 3 * rows] = ar  # decode rows
        # two pinned staging copies, used in turn: a step's update may be written
        # while the previous step's copy to the device is still in flight
        self._hosts = [host.pin_memory(), host.clone().pin_memory()]
        self._copied = [None, None]
        self._turn = 0
        self.host = self._hosts[0]
        self.dev = self.host.to(device)
        buf, r, w = self.dev, rows, width
        self.metadata = {
            "q_lens": buf[0:r], "k_lens": buf[r:2 * r], "q_starts": buf[2 * r:3 * r],
            "q_pos_offsets": buf[3 * r:4 * r], "block_table": buf[4 * r:4 * r + r * w].view(r, w),
            "block_table_row_stride": w, "total_query": r, "max_q_len": 1,
            "item_row": buf[o:o + r], "max_block_id": -1, "max_k_len": w * ops.BLOCK_SIZE,
            "decode_tokens": buf[o + r:o + 2 * r], "decode_rows": buf[o + 2 * r:o + 3 * r],
            "prefill_rows": buf[o + 3 * r:o + 3 * r], "max_prefill_q_len": 0,
        }

    def update(self, k_lens: np.ndarray, tables: np.ndarray) -> None:
        """Write this step's k_lens [rows] and block tables [rows, width] into a
        pinned staging copy (waiting, if needed, until its previous copy to the
        device has run), then copy it to the device on the current stream."""
        r, w = self.rows, self.width
        k = self._turn
        self._turn ^= 1
        if self._copied[k] is not None:
            self._copied[k].synchronize()
        self.host = self._hosts[k]
        a = self.host.numpy()
        a[r:2 * r] = k_lens
        a[3 * r:4 * r] = k_lens - 1
        a[4 * r:4 * r + r * w] = tables.reshape(-1)
        # decode items longest context first, as PackedMetadata orders them: the
        # kernel dispatches work in item order, so the short items fill its tail
        order = np.argsort(-np.asarray(k_lens, dtype=np.int64), kind="stable").astype(np.int32)
        o = 4 * r + r * w
        a[o + r:o + 2 * r] = order
        a[o + 2 * r:o + 3 * r] = order
        self.dev.copy_(self.host, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._copied[k] = ev


def metadata_from_lists(q_lens, k_lens, q_starts, q_pos_offsets, tables, device="cuda") -> dict:
    """The metadata dict from per-row host lists (one packed int32 H2D copy)."""
    return PackedMetadata(q_lens, k_lens, q_starts, q_pos_offsets, tables).upload(device)


def paged_flash_attention(q, k_cache, v_cache, metadata, num_q_heads, num_kv_heads, scale, is_causal=True):
    """Paged attention over one layer's block-structured pool.

    q: [total_query, num_q_heads, head_dim]; k_cache/v_cache: [num_blocks,
    block_size, num_kv_heads, head_dim] (not pre-gathered); metadata as built by
    build_paged_batch_metadata. Returns (o like q, l fp32 [total_query,
    num_q_heads]) where l is the log-sum-exp of the scaled scores (natural log).

    Rows with q_len == 1 go to the split-K decode kernel, rows with q_len > 1 to
    the tcgen05 chunked-prefill kernel (bf16/fp16, head_dim 64/128). A dict with
    this module's host-side row split (``prefill_rows``) is dispatched from the
    host (at head_dim 64 only when it holds no prefill row); a dict with only
    the reference builder's keys, and head_dim-64 batches with prefill rows, are
    split into decode items and prefill units on the device (one small routing
    kernel, no readback). Other dtypes and shapes run every token through the
    decode kernel, which computes any row exactly.
    """
    rows = metadata["q_lens"].shape[0]
    width = int(metadata["block_table_row_stride"])
    mbid = metadata.get("max_block_id")
    if mbid is not None and mbid >= k_cache.shape[0]:
        raise ValueError(f"paged_flash_attention: block id {mbid} outside the pool of {k_cache.shape[0]} blocks")
    mk = metadata.get("max_k_len")
    if mk is not None and mk > width * ops.BLOCK_SIZE:
        raise ValueError(f"paged_flash_attention: k_len {mk} exceeds the block table width {width} x {ops.BLOCK_SIZE}")
    o = torch.empty_like(q)
    lse = torch.empty((q.shape[0], num_q_heads), dtype=torch.float32, device=q.device)
    if rows == 0 or q.shape[0] == 0:
        return o, lse
    common = (metadata["block_table"],)
    prefill_ok = ops.prefill_supported(q, num_q_heads, num_kv_heads) and (
        o.stride(0) % 8 == 0 and o.stride(1) % 8 == 0 and o.data_ptr() % 16 == 0)
    split = "prefill_rows" in metadata and prefill_ok
    if split and q.shape[-1] == 64 and metadata["prefill_rows"].numel():
        # head_dim 64 runs one CTA per prefill unit: from the host split its grid
        # spans every row's pairs up to the longest row's, most of them empty;
        # the device router lists exactly the units the batch has.
        split = False
    if not split and prefill_ok and q.shape[0] > rows:
        # the reference builder's dict: route rows to the two kernels on the device
        return ops.paged_attention_routed(q, k_cache, v_cache, metadata["block_table"], metadata["q_lens"],
                                          metadata["k_lens"], metadata["q_starts"], metadata["q_pos_offsets"],
                                          num_q_heads, num_kv_heads, scale, is_causal, out=o, lse=lse)
    if not split:
        return ops.paged_decode(q, k_cache, v_cache, *common, metadata["q_starts"], metadata["k_lens"],
                                metadata["q_pos_offsets"], num_q_heads, num_kv_heads, scale, is_causal,
                                item_row=metadata.get("item_row"), out=o, lse=lse)
    n_dec = metadata["decode_tokens"].numel()
    n_pre = metadata["prefill_rows"].numel()
    if n_dec:
        ops.paged_decode(q, k_cache, v_cache, *common, metadata["q_starts"], metadata["k_lens"],
                         metadata["q_pos_offsets"], num_q_heads, num_kv_heads, scale, is_causal,
                         item_query=metadata["decode_tokens"], item_row=metadata["decode_rows"], out=o, lse=lse)
    if n_pre:
        ops.paged_prefill(q, k_cache, v_cache, *common, metadata["q_starts"], metadata["q_lens"], metadata["k_lens"],
                          metadata["q_pos_offsets"], num_q_heads, num_kv_heads, scale, is_causal,
                          max_q_len=metadata["max_prefill_q_len"], rows=metadata["prefill_rows"], out=o, lse=lse)
    return o, lse
