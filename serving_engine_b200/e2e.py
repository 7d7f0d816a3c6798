"""End-to-end continuous-batching driver over a Hugging Face Llama model.

The serving engine's own Scheduler / BlockManager / LLMEngine (serving_engine/
scheduler.py, block_manager.py, engine.py) stay the product path and call this
backend through the registered "paged|b200" attention function. They are not
part of this package, so this module carries a compact driver with the same
per-step semantics, used to measure end-to-end throughput and greedy-token
parity on machines where the engine package is not installed:

* running requests before waiting ones; a decode row costs one token and gets
  a new block when its table is full (block_manager.py:89-115);
* waiting requests are admitted first-come-first-served while blocks for their
  whole prompt are free and the token budget has room; prefill is chunked to
  the budget left (scheduler.py:55-149);
* one model call per step over the flattened batch: per-token write slots
  block_table[pos // 16] * 16 + pos % 16 (model_runner.py:127-129, :149-170),
  the step metadata of build_paged_batch_metadata, last-token logits per row,
  greedy argmax; a request that finished its final prefill chunk emits its
  first token (engine.py:92-116).

Unlike the reference, logits are computed for the last token of each row only
(logits_to_keep), argmax runs on the device, and all next tokens come back in
one device-to-host copy; preemption is not modelled (the pool is sized to fit).
With use_graphs, decode-only steps replay a CUDA graph captured per padded
batch-size bucket: the step's tokens, positions, slots, lengths and block
tables go to fixed device buffers in two host-to-device copies, and pad rows
attend over a reserved scratch block.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from .kv_cache import PAGED_B200_ATTN_IMPL, PagedKVCache, register
from .paged_attention import DecodeMetadataBuffer, PackedMetadata

BLOCK_SIZE = 16


@dataclass
class Seq:
    rid: int
    prompt: list
    max_new: int
    out: list = field(default_factory=list)
    table: list = field(default_factory=list)
    computed: int = 0
    prefilling: bool = True
    finished: bool = False
    tab: np.ndarray | None = None  # block table as a fixed-width int32 row (graph path)

    @property
    def total_len(self) -> int:
        return len(self.prompt) + len(self.out)


@dataclass
class StepStats:
    kind: str          # "decode", "prefill" or "mixed"
    tokens: int        # query tokens in the step
    new_tokens: int    # sampled tokens emitted
    seconds: float


class E2EEngine:
    """Continuous batching over `model` (a LlamaForCausalLM on a CUDA device)."""

    GRAPH_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256)

    def __init__(self, model, num_blocks: int, max_num_batched_tokens: int = 8192, max_num_seqs: int = 256,
                 attn_implementation: str = PAGED_B200_ATTN_IMPL, use_graphs: bool = False,
                 max_context: int = 8192):
        if attn_implementation == PAGED_B200_ATTN_IMPL:
            register()
        model.set_attn_implementation(attn_implementation)
        cfg = model.config
        self.model = model
        self.device = next(model.parameters()).device
        self.dtype = next(model.parameters()).dtype
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.kv_cache = torch.zeros(cfg.num_hidden_layers, 2, num_blocks, BLOCK_SIZE, cfg.num_key_value_heads,
                                    head_dim, dtype=self.dtype, device=self.device)
        self.cache = PagedKVCache(self.kv_cache)
        self.use_graphs = use_graphs
        self.width = -(-max_context // BLOCK_SIZE)
        # the last block is reserved as the target of padded graph rows
        self.scratch_block = num_blocks - 1 if use_graphs else None
        self.free = list(range(num_blocks - 1 if use_graphs else num_blocks))
        self.num_blocks = num_blocks
        self.graphs: dict[int, dict] = {}
        self.max_tokens = max_num_batched_tokens
        self.max_seqs = max_num_seqs
        self.waiting: list[Seq] = []
        self.running: list[Seq] = []
        self.done: list[Seq] = []
        self.stats: list[StepStats] = []
        self._next_id = 0

    def add_request(self, prompt_token_ids, max_new_tokens: int) -> int:
        s = Seq(self._next_id, list(prompt_token_ids), max_new_tokens)
        self._next_id += 1
        self.waiting.append(s)
        return s.rid

    # ----------------------------------------------------------- scheduling
    def _set_blocks(self, s: Seq, blocks) -> None:
        s.table = list(blocks)
        if self.use_graphs:
            if len(s.table) > self.width:
                raise ValueError(f"request of {s.total_len} tokens exceeds max_context {self.width * BLOCK_SIZE}")
            s.tab = np.zeros(self.width, dtype=np.int32)
            s.tab[:len(s.table)] = s.table

    def _append_block(self, s: Seq, bid: int) -> None:
        s.table.append(bid)
        if self.use_graphs:
            if len(s.table) > self.width:
                raise ValueError(f"request exceeds max_context {self.width * BLOCK_SIZE}")
            s.tab[len(s.table) - 1] = bid

    def _blocks_for(self, n_tokens: int) -> int:
        return -(-n_tokens // BLOCK_SIZE)

    def _schedule(self):
        rows = []  # (seq, chunk) ; chunk 0 = decode
        budget = self.max_tokens
        for s in self.running:
            if len(rows) >= self.max_seqs:
                break
            if s.prefilling:
                continue
            if len(s.table) * BLOCK_SIZE < s.total_len:
                if not self.free:
                    continue
                self._append_block(s, self.free.pop())
            rows.append((s, 0))
            budget -= 1
        for s in self.running:
            if len(rows) >= self.max_seqs or budget <= 0:
                break
            if s.prefilling:
                chunk = min(s.total_len - s.computed, budget)
                rows.append((s, chunk))
                budget -= chunk
        while self.waiting and len(rows) < self.max_seqs and budget > 0:
            s = self.waiting[0]
            need = self._blocks_for(s.total_len)
            if need > len(self.free):
                break
            self.waiting.pop(0)
            self._set_blocks(s, [self.free.pop() for _ in range(need)])
            self.running.append(s)
            chunk = min(s.total_len - s.computed, budget)
            rows.append((s, chunk))
            budget -= chunk
        return rows

    # ----------------------------------------------------------------- step
    @torch.inference_mode()
    def step(self) -> int:
        """One engine iteration; returns the number of tokens sampled."""
        import time

        rows = self._schedule()
        if not rows:
            return 0
        t0 = time.perf_counter()
        if self.graphs and all(c == 0 for _, c in rows) and len(rows) <= max(self.graphs):
            return self._finish_step(rows, self._graph_decode(rows), t0, len(rows))
        toks, pos, slots = [], [], []
        q_lens, k_lens, q_pos = [], [], []
        for s, chunk in rows:
            if chunk == 0:  # decode: the newest token at position total_len - 1
                p0, n = s.total_len - 1, 1
                toks.append(s.out[-1])
            else:
                p0, n = s.computed, chunk
                seq_toks = s.prompt + s.out
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
        ids = torch.from_numpy(np.asarray(toks, dtype=np.int64)).pin_memory().to(dev, non_blocking=True)
        pos_t = torch.from_numpy(np.concatenate(pos)).pin_memory().to(dev, non_blocking=True)
        slot_t = torch.from_numpy(np.concatenate(slots)).pin_memory().to(dev, non_blocking=True)
        md = PackedMetadata(q_lens, k_lens, starts, q_pos, [s.table for s, _ in rows]).upload(dev)
        last = torch.from_numpy(np.cumsum(q_lens) - 1).pin_memory().to(dev, non_blocking=True)
        out = self.model(input_ids=ids.unsqueeze(0), position_ids=pos_t.unsqueeze(0), attention_mask=None,
                         past_key_values=None, use_cache=False, cache=self.cache, write_index=slot_t,
                         paged_metadata=md, logits_to_keep=last)
        next_tok = out.logits[0].argmax(dim=-1).tolist()
        return self._finish_step(rows, next_tok, t0, len(toks))

    def _finish_step(self, rows, next_tok, t0, n_tokens) -> int:
        import time

        emitted = 0
        for (s, chunk), tok in zip(rows, next_tok):
            if chunk == 0:
                s.out.append(tok)
                emitted += 1
            else:
                s.computed += chunk
                if s.computed >= s.total_len:
                    s.prefilling = False
                    s.out.append(tok)
                    emitted += 1
            if not s.prefilling and len(s.out) >= s.max_new:
                s.finished = True
        for s, _ in rows:
            if s.finished and s in self.running:
                self.running.remove(s)
                self.free.extend(s.table)
                s.table = []
                s.tab = None
                self.done.append(s)
        kinds = {"decode" if c == 0 else "prefill" for _, c in rows}
        self.stats.append(StepStats("mixed" if len(kinds) > 1 else kinds.pop(), n_tokens, emitted,
                                    time.perf_counter() - t0))
        return emitted

    # ------------------------------------------------------------ CUDA graphs
    def _graph_inputs(self, bucket: int) -> dict:
        dev = self.device
        st = {"host": torch.zeros(3, bucket, dtype=torch.int64).pin_memory()}
        st["dev"] = st["host"].to(dev)
        st["md"] = DecodeMetadataBuffer(bucket, self.width, dev)
        st["last"] = torch.arange(bucket, device=dev)
        return st

    def _load_graph_inputs(self, st: dict, rows) -> None:
        """Real rows first, then pad rows on the scratch block."""
        b = len(rows)
        bucket = st["last"].numel()
        h = st["host"].numpy()
        k_lens = np.ones(bucket, dtype=np.int32)
        tables = np.zeros((bucket, self.width), dtype=np.int32)
        tables[:, 0] = self.scratch_block
        h[0, :] = 0
        h[1, :] = 0
        h[2, :] = self.scratch_block * BLOCK_SIZE
        for i, (s, _) in enumerate(rows):
            p = s.total_len - 1
            h[0, i] = s.out[-1]
            h[1, i] = p
            h[2, i] = s.tab[p // BLOCK_SIZE] * BLOCK_SIZE + p % BLOCK_SIZE
            k_lens[i] = s.total_len
        if b:
            tables[:b] = np.stack([s.tab for s, _ in rows])
        st["dev"].copy_(st["host"], non_blocking=True)
        st["md"].update(k_lens, tables)

    def _run_graph_body(self, st: dict):
        d = st["dev"]
        out = self.model(input_ids=d[0].unsqueeze(0), position_ids=d[1].unsqueeze(0), attention_mask=None,
                         past_key_values=None, use_cache=False, cache=self.cache, write_index=d[2],
                         paged_metadata=st["md"].metadata, logits_to_keep=st["last"])
        return out.logits[0].argmax(dim=-1)

    @torch.inference_mode()
    def capture_graphs(self, buckets=None) -> None:
        """Capture one decode-step graph per batch-size bucket (largest first, so
        the decode workspace is allocated at its largest size before capture)."""
        if not self.use_graphs:
            raise RuntimeError("engine built without use_graphs")
        buckets = sorted(buckets or [b for b in self.GRAPH_BUCKETS if b <= self.max_seqs], reverse=True)
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
            st["graph"] = g
            self.graphs[bucket] = st
        torch.cuda.synchronize(self.device)

    def _graph_decode(self, rows) -> list:
        bucket = min(b for b in self.graphs if b >= len(rows))
        st = self.graphs[bucket]
        self._load_graph_inputs(st, rows)
        st["graph"].replay()
        return st["out"][:len(rows)].tolist()

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running)

    def run(self) -> None:
        while self.has_unfinished():
            if self.step() == 0 and not self.running and self.waiting:
                raise RuntimeError("pool too small for the next request")


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


def random_llama(name: str, seed: int, dtype=torch.float32, device="cpu"):
    """Seeded random-init LlamaForCausalLM: identical weights for the same seed on
    every machine with this torch build (initialised on the CPU, then moved)."""
    from transformers import LlamaForCausalLM

    torch.manual_seed(seed)
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
