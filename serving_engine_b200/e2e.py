"""End-to-end continuous batching over a Hugging Face Llama model.

The serving engine's own Scheduler / BlockManager / LLMEngine (serving_engine/
scheduler.py, block_manager.py, engine.py) stay the product path and call this
backend through the registered "paged|b200" attention function. They are not
part of this package and cannot travel to a GPU machine without the engine
checkout, so this module carries a driver that reproduces their decisions step
for step, used to measure end-to-end throughput and to check greedy-token
parity against the reference engine's recorded runs:

* ``BlockPool`` keeps the BlockManager's rules (block_manager.py:7-141): a free
  list taken from its end, per-block reference counts, chained-hash prefix
  matching of full prompt blocks at admission, first-writer-wins registration
  of computed blocks, delta allocation of a request's whole length, one block
  per decode step when the table is full, release with hash invalidation;
* ``Scheduler`` keeps the per-step admission rules (scheduler.py:55-184):
  running requests before waiting ones, a token budget that only limits work
  piled on top of something already batched (a lone candidate always fits), the
  optional chunk floor, prefill chunks filling the budget left, and, when
  nothing at all could be scheduled while a decode row waits for a block, the
  eviction of the most recently admitted other running request (its blocks are
  freed and it is recomputed from scratch later);
* one model call per step over the flattened batch: per-token write slots
  block_table[pos // 16] * 16 + pos % 16 (model_runner.py:127-129, :149-170),
  the step metadata of build_paged_batch_metadata, greedy argmax of each row's
  last-token logits; a decode row, or a prefill row whose chunk completes its
  prompt, emits a token (engine.py:92-116).

Unlike the reference, logits are computed for the last token of each row only
(logits_to_keep), argmax runs on the device, and all next tokens come back in
one device-to-host copy. A prefill row whose whole prompt was matched in the
prefix cache (a chunk of 0 tokens) runs its last token again, which rewrites
the same K/V; the reference reads an unrelated row's logits there. With
use_graphs, decode-only steps replay a CUDA graph captured per padded
batch-size bucket: the step's positions, slots, lengths and block tables go to
fixed device buffers from pinned staging, and pad rows attend over a scratch
block placed after the engine's blocks. Such a step is launched without
waiting for it: its sampled tokens stay on the device, where the next step
gathers them as its input tokens, and reach the host (over placeholders in the
requests' outputs) while the next step runs, so the host's scheduling of step
i + 1 overlaps the GPU's step i. The schedule never needs a token value unless a
request has an end-of-sequence token, and a step with prefill rows first waits
for every pending token.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .kv_cache import PAGED_B200_ATTN_IMPL, PagedKVCache, register
from .paged_attention import DecodeMetadataBuffer, PackedMetadata

BLOCK_SIZE = 16


@dataclass
class Seq:
    """One request (serving_engine/request.py:27-64)."""

    rid: int
    prompt: list
    max_new: int
    eos: int | None = None
    out: list = field(default_factory=list)
    table: list = field(default_factory=list)
    computed: int = 0
    decoding: bool = False           # phase: prefill until its last chunk ran
    status: str = "waiting"          # waiting | running | preempted | finished
    preemptions: int = 0
    np_table: np.ndarray | None = None  # int32 copy of `table` for the graph inputs; dropped on release
    np_copied: int = 0                  # entries of `table` copied into np_table

    @property
    def total_len(self) -> int:
        return len(self.prompt) + len(self.out)

    def tokens(self) -> list:
        return self.prompt + self.out


class BlockPool:
    """Block ids, reference counts and the chained-hash prefix cache."""

    def __init__(self, num_blocks: int, block_size: int = BLOCK_SIZE):
        self.block_size = block_size
        self.free_ids = list(range(num_blocks))
        self.refs = [0] * num_blocks
        self.block_hash: list[int | None] = [None] * num_blocks
        self.by_hash: dict[int, int] = {}

    @property
    def num_free(self) -> int:
        return len(self.free_ids)

    def _take(self, s: Seq) -> None:
        bid = self.free_ids.pop()
        s.table.append(bid)
        self.refs[bid] += 1

    def match_prefix(self, s: Seq) -> None:
        """Share the cached blocks of the prompt's longest cached run of full blocks."""
        parent = None
        for i in range(len(s.prompt) // self.block_size):
            h = hash((parent, tuple(s.prompt[i * self.block_size:(i + 1) * self.block_size])))
            bid = self.by_hash.get(h)
            if bid is None:
                break
            s.table.append(bid)
            self.refs[bid] += 1
            parent = h
        s.computed = len(s.table) * self.block_size

    def shortfall(self, s: Seq) -> int:
        """Blocks still missing for the request's whole current length."""
        return -(-s.total_len // self.block_size) - len(s.table)

    def can_claim(self, s: Seq) -> bool:
        return self.shortfall(s) <= self.num_free

    def claim(self, s: Seq) -> None:
        for _ in range(self.shortfall(s)):
            self._take(s)

    def register(self, s: Seq) -> None:
        """Hash the prompt blocks that are now fully computed (first writer wins)."""
        parent = None
        for i in range(min(s.computed, len(s.prompt)) // self.block_size):
            bid = s.table[i]
            if self.block_hash[bid] is not None:
                parent = self.block_hash[bid]
                continue
            h = hash((parent, tuple(s.prompt[i * self.block_size:(i + 1) * self.block_size])))
            if h not in self.by_hash:
                self.by_hash[h] = bid
                self.block_hash[bid] = h
            parent = h

    def covers(self, s: Seq) -> bool:
        return len(s.table) * self.block_size >= s.total_len

    def can_grow(self, s: Seq) -> bool:
        return self.covers(s) or self.num_free >= 1

    def grow(self, s: Seq) -> None:
        if not self.covers(s):
            self._take(s)

    def release(self, s: Seq) -> None:
        for bid in s.table:
            self.refs[bid] -= 1
            if self.refs[bid] == 0:
                self.free_ids.append(bid)
                h = self.block_hash[bid]
                if h is not None:
                    del self.by_hash[h]
                    self.block_hash[bid] = None
        s.table = []
        s.np_table, s.np_copied = None, 0

    def preempt(self, s: Seq) -> None:
        self.release(s)
        s.computed = 0
        s.decoding = False
        s.status = "preempted"
        s.preemptions += 1


@dataclass
class StepPlan:
    rows: list = field(default_factory=list)        # (seq, chunk); chunk None = decode row
    final: set = field(default_factory=set)         # rids whose chunk completes the prefill
    preempted: list = field(default_factory=list)   # seqs evicted this step


class Scheduler:
    """Per-step admission over a BlockPool (running before waiting)."""

    def __init__(self, pool: BlockPool, max_num_batched_tokens: int | None = None,
                 max_num_seqs: int | None = None, min_chunk_size: int | None = None):
        self.pool = pool
        self.max_tokens = max_num_batched_tokens
        self.max_seqs = max_num_seqs
        self.min_chunk = min_chunk_size
        self.waiting: list[Seq] = []
        self.running: list[Seq] = []

    def add(self, s: Seq) -> None:
        self.pool.match_prefix(s)
        self.waiting.append(s)

    def _fits(self, batched: int, cost: int) -> bool:
        # the budget limits only work piled on top of something already batched
        return self.max_tokens is None or batched == 0 or batched + cost <= self.max_tokens

    def plan(self) -> StepPlan:
        plan = StepPlan()
        blocked: list[Seq] = []
        batched = 0
        for s in self.running + self.waiting:
            if self.max_seqs is not None and len(plan.rows) >= self.max_seqs:
                break
            left = s.total_len - s.computed
            if s.decoding:
                if not self._fits(batched, 1):
                    continue
                if not self.pool.can_grow(s):
                    blocked.append(s)
                    continue
                self.pool.grow(s)
                plan.rows.append((s, None))
                batched += 1
                continue
            if not self._fits(batched, left if self.min_chunk is None else min(self.min_chunk, left)):
                continue
            admitted = s.status == "running"
            if not admitted and not self.pool.can_claim(s):
                continue
            chunk = left if self.max_tokens is None else min(left, self.max_tokens - batched)
            if not admitted:
                self.pool.claim(s)
                s.status = "running"
                self.waiting = [w for w in self.waiting if w is not s]
                self.running.append(s)
            plan.rows.append((s, chunk))
            if s.computed + chunk >= s.total_len:
                plan.final.add(s.rid)
            batched += chunk
        if not plan.rows and blocked:
            # nothing advanced and a decode row waits for a block: evict the most
            # recently admitted other running request and retry the first one
            retry = blocked[0]
            victim = next((r for r in reversed(self.running) if r is not retry), None)
            if victim is not None:
                self.pool.preempt(victim)
                self.running.remove(victim)
                self.waiting.append(victim)
                plan.preempted.append(victim)
                if self.pool.can_grow(retry):
                    self.pool.grow(retry)
                    plan.rows.append((retry, None))
        return plan

    def commit(self, plan: StepPlan) -> list[Seq]:
        """Bookkeeping after the step's tokens were appended; returns the requests
        that finished."""
        finished = []
        for s, chunk in plan.rows:
            if s.out and (len(s.out) >= s.max_new or (s.eos is not None and s.out[-1] == s.eos)):
                s.status = "finished"
                self.pool.release(s)
                self.running = [r for r in self.running if r is not s]
                finished.append(s)
            elif not s.decoding:
                s.computed += chunk
                self.pool.register(s)
                if s.rid in plan.final:
                    s.decoding = True
        return finished

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running)


@dataclass
class StepStats:
    kind: str          # "decode", "prefill", "mixed" or "idle"
    tokens: int        # query tokens in the step
    new_tokens: int    # sampled tokens emitted
    seconds: float
    kv_tokens: int = 0  # keys the step's rows attend over (sum of k_len)


class E2EEngine:
    """Continuous batching over `model` (a LlamaForCausalLM on a CUDA device).

    num_blocks, max_num_batched_tokens, max_num_seqs and min_chunk_size mean what
    they mean for the reference's LLMEngine (engine.py:18-61). ``trace`` records
    every step's schedule (record_trace, on by default): per row (request id, "P"
    or "D", chunk, computed tokens before the step, block table) and the ids
    preempted. With fused_steps (bf16 / fp16 models), every step, the captured
    decode graphs included, runs the model through the fused layer kernels
    (llama_step.FusedLlamaStep) over its own weights instead of its HF modules.
    """

    GRAPH_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256)

    def __init__(self, model, num_blocks: int, max_num_batched_tokens: int | None = None,
                 max_num_seqs: int | None = None, min_chunk_size: int | None = None,
                 attn_implementation: str = PAGED_B200_ATTN_IMPL, use_graphs: bool = False,
                 max_context: int = 8192, record_logits: bool = False, record_trace: bool = True,
                 fused_steps: bool = False):
        if attn_implementation == PAGED_B200_ATTN_IMPL:
            register()
        model.set_attn_implementation(attn_implementation)
        cfg = model.config
        self.model = model
        self.device = next(model.parameters()).device
        self.dtype = next(model.parameters()).dtype
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        # with graphs, one extra block after the engine's blocks is the target of pad rows
        self.kv_cache = torch.zeros(cfg.num_hidden_layers, 2, num_blocks + (1 if use_graphs else 0), BLOCK_SIZE,
                                    cfg.num_key_value_heads, head_dim, dtype=self.dtype, device=self.device)
        self.cache = PagedKVCache(self.kv_cache)
        self.use_graphs = use_graphs
        self.width = -(-max_context // BLOCK_SIZE)
        self.scratch_block = num_blocks if use_graphs else None
        self.num_blocks = num_blocks
        self.pool = BlockPool(num_blocks)
        self.sched = Scheduler(self.pool, max_num_batched_tokens, max_num_seqs, min_chunk_size)
        self.graphs: dict[int, dict] = {}
        self.seqs: list[Seq] = []
        self.done: list[Seq] = []
        self.stats: list[StepStats] = []
        self.trace: list[dict] = []
        self.record_logits = record_logits
        self.record_trace = record_trace
        self._pending: dict | None = None  # the newest launched step whose tokens are not on the host yet
        self._eager_hosts: list | None = None  # pinned token buffers of pipelined eager steps, used in turn
        self._eager_turn = 0
        self._stage: list = [None, None]  # pinned input staging of eager steps (int64, int32), used in turn
        self._stage_ev: list = [None, None]
        self._stage_turn = 0
        # steps through the fused layer kernels instead of the HF modules
        self.fused = None
        if fused_steps:
            from .llama_step import FusedLlamaStep

            self.fused = FusedLlamaStep(model)
        self.logit_log: list[tuple] = []  # (rid, output index, top-5 ids, top-5 logits) when recording

    @property
    def free(self) -> list:
        return self.pool.free_ids

    def add_request(self, prompt_token_ids, max_new_tokens: int, eos_token_id: int | None = None) -> int:
        s = Seq(len(self.seqs), list(prompt_token_ids), max_new_tokens, eos_token_id)
        self.seqs.append(s)
        self.sched.add(s)
        return s.rid

    # ----------------------------------------------------------------- step
    @torch.inference_mode()
    def step(self) -> int:
        """One engine iteration; returns the number of tokens sampled."""
        t0 = time.perf_counter()
        plan = self.sched.plan()
        if self.record_trace:
            self.trace.append({
                "rows": [[s.rid, "D" if c is None else "P", 0 if c is None else c, s.computed, list(s.table)]
                         for s, c in plan.rows],
                "preempted": [s.rid for s in plan.preempted]})
        if not plan.rows:
            self.stats.append(StepStats("idle", 0, 0, time.perf_counter() - t0))
            return 0
        n_tokens = sum(1 if c is None else max(c, 1) for _, c in plan.rows)
        kv_tokens = sum(s.total_len if c is None else max(s.computed + c, 1) for s, c in plan.rows)
        previous = self._pending
        if (self.graphs and not self.record_logits and all(c is None for _, c in plan.rows)
                and len(plan.rows) <= max(self.graphs)):
            # decode-only step: launched without waiting; its tokens stay on the
            # device (the next step reads them there) and reach the host while the
            # next step runs
            self._graph_decode(plan.rows, previous)
            if any(s.eos is not None for s, _ in plan.rows):
                self._drain()  # the end-of-sequence check below needs the values
            emitted = len(plan.rows)
        elif self._can_pipeline(plan):
            # eager step launched without waiting, like the graph steps: a row whose
            # newest token the previous step produced takes it on the device, and
            # this step's tokens reach the host while the next step's inputs are
            # prepared and launched
            emitted = self._eager_launch(plan, previous)
        else:
            self._drain()  # a prefill row may need the real values of earlier tokens
            previous = None
            next_tok = self._eager_step(plan.rows).tolist()
            emitted = 0
            for (s, c), tok in zip(plan.rows, next_tok):
                if c is None or s.rid in plan.final:
                    s.out.append(int(tok))
                    emitted += 1
        for s in self.sched.commit(plan):
            self.done.append(s)
        if previous is not None and previous is not self._pending:
            self._drain(previous)
        if self._pending is not None and not self.sched.has_unfinished():
            self._drain()  # nothing left to run: the caller may read every output now
        kinds = {"decode" if c is None else "prefill" for _, c in plan.rows}
        self.stats.append(StepStats("mixed" if len(kinds) > 1 else kinds.pop(), n_tokens, emitted,
                                    time.perf_counter() - t0, kv_tokens))
        return emitted

    def _drain(self, pending: dict | None = None) -> None:
        """Wait for a launched step's tokens (default: the newest) and write them
        over its placeholders (rows whose index is None sampled nothing)."""
        pending = self._pending if pending is None else pending
        if pending is None:
            return
        pending["event"].synchronize()
        values = pending["host"][:len(pending["rows"])].tolist()
        for (s, idx), v in zip(pending["rows"], values):
            if idx is not None:
                s.out[idx] = v
        if pending is self._pending:
            self._pending = None

    def _can_pipeline(self, plan: StepPlan) -> bool:
        """An eager step may run ahead of the host when no value of a sampled token
        is needed before it runs: no logits are recorded, no row stops at an
        end-of-sequence token, and no prefill chunk re-reads an output token whose
        value is still on the device (a recomputed, preempted request)."""
        if self.record_logits:
            return False
        for s, c in plan.rows:
            if s.eos is not None or (c is not None and c > 0 and None in s.out):
                return False
        return True

    def _eager_launch(self, plan: StepPlan, previous: dict | None) -> int:
        """Launch an eager step and leave its tokens pending (placeholders in each
        sampling row's output); returns the number of tokens sampled."""
        rows = plan.rows
        nxt = self._eager_step(rows, previous)
        n = len(rows)
        if self._eager_hosts is None or self._eager_hosts[0].numel() < n:
            self._eager_hosts = [torch.zeros(max(n, 256), dtype=torch.int64).pin_memory() for _ in range(2)]
        host = self._eager_hosts[self._eager_turn]
        self._eager_turn ^= 1
        host[:n].copy_(nxt, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        placed, emitted = [], 0
        for s, c in rows:
            if c is None or s.rid in plan.final:
                placed.append((s, len(s.out)))
                s.out.append(None)
                emitted += 1
            else:
                placed.append((s, None))
        self._pending = {"rows": placed, "host": host, "event": ev, "st": {"out": nxt},
                         "row_of": {s.rid: i for i, (s, _) in enumerate(rows)}}
        return emitted

    def _staging(self, n64: int, n32: int) -> tuple:
        """The next pinned staging set (int64 and int32 buffers of at least n64 and
        n32 elements), once the copies that last read it have run."""
        k = self._stage_turn
        self._stage_turn ^= 1
        if self._stage_ev[k] is not None:
            self._stage_ev[k].synchronize()
        st = self._stage[k]
        if st is None or st[0].numel() < n64 or st[1].numel() < n32:
            c64 = max(n64, 2 * st[0].numel() if st is not None else 0, 1 << 16)
            c32 = max(n32, 2 * st[1].numel() if st is not None else 0, 1 << 16)
            st = (torch.empty(c64, dtype=torch.int64).pin_memory(), torch.empty(c32, dtype=torch.int32).pin_memory())
            self._stage[k] = st
        return st

    def _eager_step(self, rows, previous: dict | None = None) -> torch.Tensor:
        """One step through the model with host-built inputs; returns the greedy
        token of each row's last position, on the device. A decode row whose
        newest token is a placeholder of `previous` (a launched step) takes its
        value from that step's device output."""
        toks, pos, slots = [], [], []
        q_lens, k_lens, q_pos = [], [], []
        gather = []  # (token index, row of the previous step's output)
        for s, chunk in rows:
            seq_toks = s.tokens()
            if chunk is None or chunk == 0:  # the newest token (a decode row, or a fully cached prompt)
                p0, n = s.total_len - 1, 1
                t = seq_toks[-1]
                if t is None:
                    gather.append((len(toks), previous["row_of"][s.rid]))
                    t = 0
                toks.append(t)
            else:
                p0, n = s.computed, chunk
                toks.extend(seq_toks[p0:p0 + n])
            positions = np.arange(p0, p0 + n)
            table = np.asarray(s.table, dtype=np.int64)
            pos.append(positions)
            slots.append(table[positions // BLOCK_SIZE] * BLOCK_SIZE + positions % BLOCK_SIZE)
            q_lens.append(n)
            k_lens.append(p0 + n)
            q_pos.append(p0)
        starts = np.concatenate(([0], np.cumsum(q_lens)[:-1])).tolist()
        dev = self.device
        packed = PackedMetadata(q_lens, k_lens, starts, q_pos, [s.table for s, _ in rows])
        # token ids, positions, slots, last-token indices and (when needed) the
        # gather rows in one int64 staging buffer, the metadata in an int32 one:
        # two pinned sets used in turn, each rewritten only once its previous
        # copies have run (a launched step may still be reading the other set)
        nt, nr = len(toks), len(rows)
        n64 = 4 * nt + nr
        st64, st32 = self._staging(n64, packed.host.numel())
        a = st64.numpy()
        a[0:nt] = toks
        a[nt:2 * nt] = np.concatenate(pos)
        a[2 * nt:3 * nt] = np.concatenate(slots)
        a[3 * nt:3 * nt + nr] = np.cumsum(q_lens) - 1
        if gather:
            src = a[3 * nt + nr:n64]
            src[:] = -1
            for ti, pi in gather:
                src[ti] = pi
        d64 = st64[:n64].to(dev, non_blocking=True)
        md = packed.upload(dev, staging=st32)
        self._stage_ev[self._stage_turn ^ 1] = torch.cuda.Event()
        self._stage_ev[self._stage_turn ^ 1].record()
        ids, pos_t, slot_t = d64[0:nt], d64[nt:2 * nt], d64[2 * nt:3 * nt]
        last = d64[3 * nt:3 * nt + nr]
        if gather:
            src_t = d64[3 * nt + nr:n64]
            picked = previous["st"]["out"].index_select(0, src_t.clamp(min=0))
            ids = torch.where(src_t >= 0, picked, ids)
        if self.fused is not None:
            logits = self.fused.logits(ids, pos_t, slot_t, self.kv_cache, md, last)
        else:
            out = self.model(input_ids=ids.unsqueeze(0), position_ids=pos_t.unsqueeze(0), attention_mask=None,
                             past_key_values=None, use_cache=False, cache=self.cache, write_index=slot_t,
                             paged_metadata=md, logits_to_keep=last)
            logits = out.logits[0]
        if self.record_logits:
            top = torch.topk(logits.float(), 5, dim=-1)
            ids5, vals5 = top.indices.tolist(), top.values.tolist()
            for i, (s, c) in enumerate(rows):
                if c is None or (s.computed + c >= s.total_len):
                    self.logit_log.append((s.rid, len(s.out), ids5[i], vals5[i]))
        return logits.argmax(dim=-1)

    # ------------------------------------------------------------ CUDA graphs
    def _graph_inputs(self, bucket: int) -> dict:
        """Fixed device buffers a bucket's graph reads: rows 0-2 of ``dev`` are the
        tokens, positions and write slots. Host staging is pinned and used in
        turn (``host``: tokens, positions, slots and, in row 3, where each token
        comes from: -1 for the host value, else its row in the previous step's
        device output)."""
        dev = self.device
        st = {"hosts": [torch.zeros(4, bucket, dtype=torch.int64).pin_memory() for _ in range(2)],
              "copied": [None, None], "turn": 0}
        st["host"] = st["hosts"][0]
        st["dev"] = torch.zeros(3, bucket, dtype=torch.int64, device=dev)
        st["src"] = torch.zeros(bucket, dtype=torch.int64, device=dev)
        st["md"] = DecodeMetadataBuffer(bucket, self.width, dev)
        st["last"] = torch.arange(bucket, device=dev)
        st["tokens_host"] = [torch.zeros(bucket, dtype=torch.int64).pin_memory() for _ in range(2)]
        return st

    def _np_table(self, s: Seq) -> np.ndarray:
        """The request's block table as int32, copied incrementally: a table only
        grows by appends until BlockPool.release empties it (and drops the copy)."""
        n = len(s.table)
        if n > self.width:
            raise ValueError(f"request of {s.total_len} tokens exceeds max_context {self.width * BLOCK_SIZE}")
        if s.np_table is None:
            s.np_table = np.zeros(self.width, dtype=np.int32)
            s.np_copied = 0
        if s.np_copied < n:
            s.np_table[s.np_copied:n] = s.table[s.np_copied:n]
            s.np_copied = n
        return s.np_table

    def _load_graph_inputs(self, st: dict, rows, previous: dict | None = None) -> None:
        """Real rows first, then pad rows on the scratch block. A row whose newest
        token is still a placeholder of the previous (graph) step takes it from
        that step's device output."""
        bucket = st["last"].numel()
        b = len(rows)
        k = st["turn"]
        st["turn"] ^= 1
        if st["copied"][k] is not None:
            st["copied"][k].synchronize()  # its previous copy to the device has run
        st["host"] = st["hosts"][k]
        h = st["host"].numpy()
        k_lens = np.ones(bucket, dtype=np.int32)
        tables = np.zeros((bucket, self.width), dtype=np.int32)
        tables[b:, 0] = self.scratch_block
        h[:, b:] = 0
        h[2, b:] = self.scratch_block * BLOCK_SIZE
        h[3, :] = -1
        gather = False
        if b:
            seqs = [s for s, _ in rows]
            tot = np.fromiter((s.total_len for s in seqs), dtype=np.int64, count=b)
            pos = tot - 1
            for i, s in enumerate(seqs):
                tables[i] = self._np_table(s)
            blk = tables[np.arange(b), pos // BLOCK_SIZE].astype(np.int64)
            prev_row = previous["row_of"] if previous is not None else {}
            toks = np.empty(b, dtype=np.int64)
            for i, s in enumerate(seqs):
                t = s.out[-1]
                if t is None:  # produced by the previous step, still on the device
                    h[3, i] = prev_row[s.rid]
                    toks[i] = 0
                    gather = True
                else:
                    toks[i] = t
            h[0, :b] = toks
            h[1, :b] = pos
            h[2, :b] = blk * BLOCK_SIZE + pos % BLOCK_SIZE
            k_lens[:b] = tot
        st["dev"].copy_(st["host"][:3], non_blocking=True)
        if gather:
            st["src"].copy_(st["host"][3], non_blocking=True)
            picked = previous["st"]["out"].index_select(0, st["src"].clamp(min=0))
            st["dev"][0].copy_(torch.where(st["src"] >= 0, picked, st["dev"][0]))
        ev = torch.cuda.Event()
        ev.record()
        st["copied"][k] = ev
        st["md"].update(k_lens, tables)

    def _run_graph_body(self, st: dict):
        d = st["dev"]
        if self.fused is not None:
            return self.fused.logits(d[0], d[1], d[2], self.kv_cache, st["md"].metadata).argmax(dim=-1)
        out = self.model(input_ids=d[0].unsqueeze(0), position_ids=d[1].unsqueeze(0), attention_mask=None,
                         past_key_values=None, use_cache=False, cache=self.cache, write_index=d[2],
                         paged_metadata=st["md"].metadata, logits_to_keep=st["last"])
        return out.logits[0].argmax(dim=-1)

    @torch.inference_mode()
    def capture_graphs(self, buckets=None) -> None:
        """Capture one decode-step graph per batch-size bucket (largest first, so
        the decode workspace is allocated at its largest size before capture),
        and replay each once: the first launch of an instantiated graph uploads
        it to the device (tens of milliseconds for the 256-row step), which
        belongs to start-up, not to the first decode step. The replay runs pad
        rows only, whose KV writes land on the scratch block."""
        if not self.use_graphs:
            raise RuntimeError("engine built without use_graphs")
        limit = self.sched.max_seqs or max(self.GRAPH_BUCKETS)
        buckets = sorted(buckets or [b for b in self.GRAPH_BUCKETS if b <= limit], reverse=True)
        pool = torch.cuda.graph_pool_handle()
        side = torch.cuda.Stream(device=self.device)
        for bucket in buckets:
            st = self._graph_inputs(bucket)
            self._load_graph_inputs(st, [])
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._run_graph_body(st)
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                st["out"] = self._run_graph_body(st)
            g.replay()
            st["graph"] = g
            self.graphs[bucket] = st
        torch.cuda.synchronize(self.device)

    def _graph_decode(self, rows, previous: dict | None) -> None:
        """Replay the bucket's graph for a decode-only step without waiting for it:
        each row gets a placeholder token, filled in by _drain once the step's
        tokens are on the host."""
        bucket = min(b for b in self.graphs if b >= len(rows))
        st = self.graphs[bucket]
        self._load_graph_inputs(st, rows, previous)
        st["graph"].replay()
        host = st["tokens_host"][st["turn"]]
        host[:len(rows)].copy_(st["out"][:len(rows)], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        placed = []
        for s, _ in rows:
            placed.append((s, len(s.out)))
            s.out.append(None)
        self._pending = {"rows": placed, "host": host, "event": ev, "st": st,
                         "row_of": {s.rid: i for i, (s, _) in enumerate(rows)}}

    def has_unfinished(self) -> bool:
        return self.sched.has_unfinished()

    def run(self, max_idle_steps: int = 1000) -> None:
        idle = 0
        while self.has_unfinished():
            if self.step() == 0 and self.stats[-1].kind == "idle":
                idle += 1
                if idle > max_idle_steps:
                    raise RuntimeError("no request can be scheduled: the pool is too small")
            else:
                idle = 0


def llama_config(name: str):
    """The model shapes of the end-to-end configurations (random-init weights)."""
    from transformers import LlamaConfig

    if name == "config4":
        return LlamaConfig(hidden_size=2048, intermediate_size=8192, num_hidden_layers=16, num_attention_heads=32,
                           num_key_value_heads=8, head_dim=64, vocab_size=32000, rope_theta=10000.0,
                           max_position_embeddings=8192, hidden_act="silu", tie_word_embeddings=False)
    if name == "tiny":
        return LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                           num_key_value_heads=2, head_dim=64, vocab_size=1000, rope_theta=10000.0,
                           max_position_embeddings=1024, hidden_act="silu", tie_word_embeddings=False)
    raise ValueError(name)


def random_llama(name: str, seed: int, dtype=torch.float32, device="cpu", init_on_device: bool = False):
    """Seeded random-init LlamaForCausalLM. By default the weights are initialised
    on the CPU, then moved: identical weights for the same seed on every machine
    with this torch build (what the parity fixtures rely on). init_on_device
    initialises directly on `device` (much faster for the large shapes; other
    values than the CPU initialisation gives)."""
    from transformers import LlamaForCausalLM

    torch.manual_seed(seed)
    if init_on_device:
        torch.cuda.manual_seed(seed)
        with torch.device(device):
            model = LlamaForCausalLM(llama_config(name))
        return model.to(dtype=dtype).eval()
    model = LlamaForCausalLM(llama_config(name))
    return model.to(device=device, dtype=dtype).eval()


def config4_requests(seed: int = 0, n: int = 256, vocab: int = 32000):
    """256 prompts: token ids U[0, vocab), lengths lognormal with median 512 and
    the workload generator's default spread (cv = 1 -> sigma = sqrt(ln 2);
    serving_engine/workload.py:24-33), clipped to [32, 4096]."""
    rng = np.random.default_rng(seed)
    sigma = math.sqrt(math.log(2.0))
    lens = np.clip(np.round(np.exp(rng.normal(math.log(512.0), sigma, size=n))), 32, 4096).astype(int)
    return [rng.integers(0, vocab, size=int(k)).tolist() for k in lens]
