"""Generate the golden fixtures in tests/golden/ by running the REFERENCE itself.

Run in a container where the reference checkout is importable:

    python tests/golden/make_golden.py --reference /path/to/serving-engine

It imports the reference package (serving_engine.*) and its third-party
oracle (transformers' eager_paged_attention_forward) and records:

* attention outputs of seeded batches through
  - the reference's eager oracle path: _PagedKVCache.update
    (model_runner.py:34-40) + eager_paged_attention_forward with the additive
    mask built as model_runner.py:185-207 builds it;
  - the reference's Triton kernel paged_flash_attention
    (paged_attention_kernel.py:125-160) under TRITON_INTERPRET=1 (fp32 only:
    the interpreter mishandles bf16 on CPU), which also yields the LSE and the
    is_causal=False behaviour;
* the pool after _PagedKVCache.write (index_copy_) of strided K/V views;
* build_paged_batch_metadata outputs and per-token write slots
  (ModelRunner._flat_slot) over a scripted run of the reference
  Scheduler/BlockManager with chunked prefill, decode and prefix sharing;
* greedy tokens of the reference engine itself (fp32, CPU) on a tiny random
  Llama, and on the config-4 model shape with a reduced workload whose
  schedule has chunked prefill, prefix-cache hits and a preemption: its
  per-step schedule and the top-5 logits behind every sampled token too.

``--only PART`` regenerates just that part and keeps the other fixtures.

Inputs are regenerated in the tests from the same seeds
(serving_engine_b200.workloads); their sha256 is stored to prove it.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import types
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from serving_engine_b200.workloads import PagedBatch  # noqa: E402
from tests.golden.cases import attention_batches, digest, kv_append_inputs, noncausal_batch  # noqa: E402


def eager_reference(b: PagedBatch, dtype: torch.dtype) -> torch.Tensor:
    """The reference's eager oracle path on batch b, writing each query token's own
    K/V (already in the pool) through _PagedKVCache.update first."""
    from transformers.integrations.eager_paged import eager_paged_attention_forward

    from serving_engine.model_runner import _PagedKVCache

    hkv, d = b.num_kv_heads, b.head_dim
    kv = torch.stack([b.k_cache, b.v_cache]).unsqueeze(0).to(dtype).clone()
    cache = _PagedKVCache(kv)
    write, q_group, q_pos, read, k_pos, k_group = [], [], [], [], [], []
    for r, bt in enumerate(b.block_tables):
        for i in range(b.q_lens[r]):
            p = b.q_pos_offsets[r] + i
            write.append(bt[p // 16] * 16 + p % 16)
            q_group.append(r)
            q_pos.append(p)
        for p in range(b.k_lens[r]):
            read.append(bt[p // 16] * 16 + p % 16)
            k_pos.append(p)
            k_group.append(r)
    write_t, read_t = torch.tensor(write), torch.tensor(read)
    k_flat = kv[0, 0].view(-1, hkv, d)
    v_flat = kv[0, 1].view(-1, hkv, d)
    key = k_flat[write_t].transpose(0, 1).unsqueeze(0).clone()
    value = v_flat[write_t].transpose(0, 1).unsqueeze(0).clone()
    allowed = (torch.tensor(q_group)[:, None] == torch.tensor(k_group)[None, :]) & (
        torch.tensor(k_pos)[None, :] <= torch.tensor(q_pos)[:, None])
    mask = torch.zeros(len(q_pos), len(read), dtype=dtype)
    mask.masked_fill_(~allowed, torch.finfo(dtype).min)
    module = types.SimpleNamespace(layer_idx=0, num_key_value_groups=b.num_q_heads // hkv)
    query = b.q.to(dtype).transpose(0, 1).unsqueeze(0)
    out, _ = eager_paged_attention_forward(module, query, key, value, mask[None, None], b.scale,
                                           cache=cache, read_index=read_t, write_index=write_t)
    return out[0]


def triton_reference(b: PagedBatch, is_causal: bool = True):
    from serving_engine.paged_attention_kernel import paged_flash_attention

    md = b.metadata("cpu")
    return paged_flash_attention(b.q, b.k_cache, b.v_cache, md, b.num_q_heads, b.num_kv_heads, b.scale,
                                 is_causal=is_causal)


def attention_cases(out: dict, meta: dict) -> None:
    for name, (b, run_triton) in attention_batches().items():
        meta[name] = {"q": digest(b.q), "k_cache": digest(b.k_cache), "v_cache": digest(b.v_cache)}
        out[f"{name}__eager"] = eager_reference(b, b.q.dtype).float().numpy()
        if b.q.dtype != torch.float32:
            out[f"{name}__eager_fp32"] = eager_reference(b, torch.float32).numpy()
        if run_triton:
            o, l = triton_reference(b, True)
            out[f"{name}__triton_o"] = o.float().numpy()
            out[f"{name}__triton_lse"] = l.numpy()
        print(name, "done", flush=True)
    # is_causal=False: only the Triton kernel defines it (zero-padded keys of the
    # last block then enter the softmax with score 0).
    b = noncausal_batch()
    meta["noncausal_fp32"] = {"q": digest(b.q), "k_cache": digest(b.k_cache), "v_cache": digest(b.v_cache)}
    o, l = triton_reference(b, False)
    out["noncausal_fp32__triton_o"] = o.numpy()
    out["noncausal_fp32__triton_lse"] = l.numpy()


def kv_append_case(out: dict, meta: dict) -> None:
    """_PagedKVCache.write on HF-layout [1, HKV, S, D] views (transposes of [1, S, HKV, D])."""
    from serving_engine.model_runner import _PagedKVCache

    for dtype, tag in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        kv, k_src, v_src, slots = kv_append_inputs(dtype)
        nb, hkv, d = kv.shape[2], kv.shape[4], kv.shape[5]
        meta[f"kv_append_{tag}"] = {"kv": digest(kv), "k": digest(k_src), "v": digest(v_src),
                                    "slots": slots.tolist()}
        cache = _PagedKVCache(kv)
        cache.write(k_src.transpose(1, 2), v_src.transpose(1, 2), 1, slots)
        meta[f"kv_append_{tag}"]["pool_after"] = digest(kv)
        flat = kv[1].reshape(2, nb * 16, hkv, d)
        out[f"kv_append_{tag}__written"] = flat[:, slots].float().numpy()


def scheduler_trace(meta: dict) -> None:
    """Drive the reference Scheduler/BlockManager (no model) and record the
    metadata the reference builder produces at each step."""
    from serving_engine.block_manager import BlockManager
    from serving_engine.model_runner import ModelRunner
    from serving_engine.paged_attention_kernel import build_paged_batch_metadata
    from serving_engine.request import Request, RequestPhase
    from serving_engine.scheduler import Scheduler

    bm = BlockManager(num_gpu_blocks=48, block_size=16)
    sched = Scheduler(bm, max_num_batched_tokens=64, max_num_seqs=6, min_chunk_size=8)
    shared = list(range(1000, 1040))
    prompts = [shared + list(range(7)), list(range(2000, 2070)), list(range(3000, 3016)), shared + [5, 6, 7]]
    reqs = [Request(request_id=f"r{i}", prompt_token_ids=p, max_new_tokens=3 + i) for i, p in enumerate(prompts)]
    runner = object.__new__(ModelRunner)
    runner.block_size = 16
    steps = []
    arrivals = {0: [0, 1], 2: [2], 4: [3]}
    for step in range(40):
        for i in arrivals.get(step, []):
            sched.add_request(reqs[i])
        if not sched.has_unfinished_requests():
            break
        so = sched.schedule()
        if not so.scheduled_requests:
            continue
        rows = []
        writes = []
        for req in so.scheduled_requests:
            prefill = req.phase == RequestPhase.NEEDS_PREFILL
            row = {"phase": "NEEDS_PREFILL" if prefill else "NEEDS_DECODE",
                   "chunk": so.prefill_chunk_sizes.get(req.request_id, 0),
                   "num_computed_tokens": req.num_computed_tokens, "total_len": req.total_len,
                   "block_table": list(req.block_table)}
            rows.append(row)
            positions = (range(req.num_computed_tokens, req.num_computed_tokens + row["chunk"]) if prefill
                         else [req.total_len - 1])
            writes.extend(runner._flat_slot(req.block_table, p) for p in positions)
        md = build_paged_batch_metadata(so, device="cpu")
        steps.append({
            "rows": rows,
            "write_index": writes,
            "metadata": {k: (v.tolist() if isinstance(v, torch.Tensor) else v) for k, v in md.items()},
        })
        # engine.step bookkeeping (engine.py:106-115) with a made-up sampled token
        for req in so.scheduled_requests:
            if req.phase == RequestPhase.NEEDS_DECODE or req.request_id in so.prefill_final_chunk:
                req.output_token_ids.append(7)
        sched.update_after_step(so)
    meta["scheduler_trace"] = steps


def e2e_trace(meta: dict) -> None:
    """Greedy tokens of the reference engine itself (LLMEngine + Scheduler +
    BlockManager + ModelRunner.forward, eager paged attention, fp32, CPU) on a
    seeded tiny random Llama, with chunked prefill forced by a small budget."""
    from serving_engine.block import BLOCK_SIZE
    from serving_engine.block_manager import BlockManager
    from serving_engine.engine import LLMEngine
    from serving_engine.model_runner import ModelRunner
    from serving_engine.scheduler import Scheduler

    from serving_engine_b200.e2e import random_llama
    from tests.golden.cases import e2e_prompts

    model = random_llama("tiny", seed=0)
    cfg = model.config
    runner = object.__new__(ModelRunner)
    runner.device = "cpu"
    runner.dtype = torch.float32
    runner.attn_implementation = "paged|eager"
    runner.model = model
    runner.model.set_attn_implementation("paged|eager")
    runner.block_size = BLOCK_SIZE
    runner.num_gpu_blocks = 64
    runner.tokenizer = None
    runner.kv_cache = torch.zeros(cfg.num_hidden_layers, 2, 64, BLOCK_SIZE, cfg.num_key_value_heads, cfg.head_dim)
    engine = object.__new__(LLMEngine)
    engine.model_runner = runner
    engine.block_manager = BlockManager(64, BLOCK_SIZE)
    engine.scheduler = Scheduler(engine.block_manager, max_num_batched_tokens=32)
    engine.requests = {}
    prompts, max_new = e2e_prompts()
    ids = [engine.add_request(prompt_token_ids=p, max_new_tokens=max_new, ignore_eos=True) for p in prompts]
    steps = 0
    while engine.scheduler.has_unfinished_requests():
        engine.step()
        steps += 1
    meta["e2e_tiny_fp32"] = {"outputs": [engine.requests[r].output_token_ids for r in ids], "steps": steps,
                             "max_num_batched_tokens": 32, "num_gpu_blocks": 64, "model": "tiny", "seed": 0}


def e2e_config4_trace(out: dict, meta: dict) -> None:
    """The reference engine (LLMEngine + Scheduler + BlockManager +
    ModelRunner.forward, eager paged attention, fp32, CPU) on the config-4 model
    shape with the reduced workload of cases.e2e_config4_workload: requests
    arrive at their listed steps, and each step is engine.step() (engine.py:92-116)
    written out, as the reference's own scripts/diagnose_triton_kernel_divergence.py
    does, so the logits behind every sampled token can be kept. Records the
    schedule of every step (rows: request index, phase, chunk, computed tokens,
    block table; preempted request indices), the greedy tokens, and per sampled
    token its top-5 token ids and logits."""
    from serving_engine.block import BLOCK_SIZE
    from serving_engine.block_manager import BlockManager
    from serving_engine.engine import LLMEngine
    from serving_engine.model_runner import ModelRunner
    from serving_engine.request import RequestPhase
    from serving_engine.scheduler import Scheduler

    from serving_engine_b200.e2e import random_llama
    from tests.golden.cases import e2e_config4_workload

    w = e2e_config4_workload()
    model = random_llama(w["model"], seed=w["seed"])
    cfg = model.config
    nb = w["num_gpu_blocks"]
    runner = object.__new__(ModelRunner)
    runner.device = "cpu"
    runner.dtype = torch.float32
    runner.attn_implementation = "paged|eager"
    runner.model = model
    runner.model.set_attn_implementation("paged|eager")
    runner.block_size = BLOCK_SIZE
    runner.num_gpu_blocks = nb
    runner.tokenizer = None
    runner.kv_cache = torch.zeros(cfg.num_hidden_layers, 2, nb, BLOCK_SIZE, cfg.num_key_value_heads, cfg.head_dim)
    engine = object.__new__(LLMEngine)
    engine.model_runner = runner
    engine.block_manager = BlockManager(nb, BLOCK_SIZE)
    engine.scheduler = Scheduler(engine.block_manager, max_num_batched_tokens=w["max_num_batched_tokens"],
                                 max_num_seqs=w["max_num_seqs"], min_chunk_size=w["min_chunk_size"])
    engine.requests = {}
    index = {}
    trace, sampled, top_ids, top_vals = [], [], [], []
    step = 0
    last_arrival = max(w["arrivals"])
    while True:
        for i in w["arrivals"].get(step, []):
            rid = engine.add_request(prompt_token_ids=w["prompts"][i], max_new_tokens=w["max_new"], ignore_eos=True)
            index[rid] = i
        if not engine.scheduler.has_unfinished_requests() and step > last_arrival:
            break
        so = engine.scheduler.schedule()
        step += 1
        trace.append({"rows": [[index[r.request_id], "P" if r.phase == RequestPhase.NEEDS_PREFILL else "D",
                                so.prefill_chunk_sizes.get(r.request_id, 0), r.num_computed_tokens,
                                list(r.block_table)] for r in so.scheduled_requests],
                      "preempted": [index[r.request_id] for r in so.preempted_requests]})
        if not so.scheduled_requests:
            continue
        logits = engine.model_runner.forward(so)
        next_tokens = logits.argmax(dim=-1)
        top = torch.topk(logits.float(), 5, dim=-1)
        for j, (req, tok) in enumerate(zip(so.scheduled_requests, next_tokens)):
            if req.phase == RequestPhase.NEEDS_DECODE or req.request_id in so.prefill_final_chunk:
                sampled.append([index[req.request_id], req.output_len])
                top_ids.append(top.indices[j].tolist())
                top_vals.append(top.values[j].tolist())
                req.output_token_ids.append(tok.item())
        engine.scheduler.update_after_step(so)
        print("e2e config4 step", step, flush=True)
    outputs = [None] * len(w["prompts"])
    for rid, i in index.items():
        outputs[i] = engine.requests[rid].output_token_ids
    vals = np.asarray(top_vals, dtype=np.float32)
    meta["e2e_config4_fp32"] = {"outputs": outputs, "trace": trace, "steps": step, "sampled": sampled,
                                "min_top1_margin": float((vals[:, 0] - vals[:, 1]).min()),
                                "preemptions": sum(len(t["preempted"]) for t in trace)}
    out["e2e_config4_fp32__top5_ids"] = np.asarray(top_ids, dtype=np.int32)
    out["e2e_config4_fp32__top5_logits"] = vals


PARTS = ("attention", "kv_append", "scheduler_trace", "e2e_tiny", "e2e_config4")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SEB_REFERENCE", "/root/reference"))
    ap.add_argument("--only", choices=PARTS, action="append",
                    help="regenerate only these parts and keep the rest of the existing fixtures")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    parts = set(args.only or PARTS)
    arrays, meta = {}, {}
    if args.only:
        arrays = dict(np.load(HERE / "golden.npz"))
        meta = json.loads((HERE / "golden.json").read_text())
    if "attention" in parts:
        attention_cases(arrays, meta)
    if "kv_append" in parts:
        kv_append_case(arrays, meta)
    if "scheduler_trace" in parts:
        scheduler_trace(meta)
    if "e2e_tiny" in parts:
        e2e_trace(meta)
    if "e2e_config4" in parts:
        e2e_config4_trace(arrays, meta)
    import transformers
    meta["_generated_with"] = {"torch": torch.__version__, "transformers": transformers.__version__,
                               "numpy": np.__version__}
    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "golden.npz", HERE / "golden.json")


if __name__ == "__main__":
    main()
