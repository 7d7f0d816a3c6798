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
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from .kv_cache import PAGED_B200_ATTN_IMPL, PagedKVCache, register
from .paged_attention import PackedMetadata

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

    def __init__(self, model, num_blocks: int, max_num_batched_tokens: int = 8192, max_num_seqs: int = 256,
                 attn_implementation: str = PAGED_B200_ATTN_IMPL):
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
        self.free = list(range(num_blocks))
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
                s.table.append(self.free.pop())
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
            s.table = [self.free.pop() for _ in range(need)]
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
                self.done.append(s)
        kinds = {"decode" if c == 0 else "prefill" for _, c in rows}
        self.stats.append(StepStats("mixed" if len(kinds) > 1 else kinds.pop(), len(toks), emitted,
                                    time.perf_counter() - t0))
        return emitted

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
