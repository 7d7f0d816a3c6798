"""The end-to-end driver's Scheduler / BlockPool against schedules the
reference's own Scheduler / BlockManager produced (tests/golden, recorded by
make_golden.py from serving_engine/scheduler.py and block_manager.py): the
same rows in the same order, the same chunks, computed-token counts and block
tables at every step, and the same preemptions. The schedule does not depend
on token values (no EOS), so no model is needed; the config-4 run also feeds
the reference's sampled tokens back, as the engine would."""
from serving_engine_b200.e2e import BlockPool, Scheduler, Seq
from tests.golden.cases import e2e_config4_workload


def run_schedule(prompts, max_new, num_blocks, budget, max_seqs, min_chunk, arrivals, tokens=None,
                 max_steps=3000, skip_empty=False, step_limit=None):
    """Drive the Scheduler like the engine loop; returns per-step records."""
    sched = Scheduler(BlockPool(num_blocks), budget, max_seqs, min_chunk)
    seqs = [Seq(i, list(p), max_new) for i, p in enumerate(prompts)]
    trace, step = [], 0
    last = max(arrivals)
    while step < max_steps and (step_limit is None or step < step_limit):
        for i in arrivals.get(step, []):
            sched.add(seqs[i])
        if not sched.has_unfinished() and (step > last or step_limit is not None):
            break
        plan = sched.plan()
        step += 1
        if skip_empty and not plan.rows:
            continue
        trace.append((plan, [(s, c, s.computed, s.total_len, list(s.table)) for s, c in plan.rows]))
        for s, c in plan.rows:
            if c is None or s.rid in plan.final:
                s.out.append(7 if tokens is None else tokens[s.rid][len(s.out)])
        sched.commit(plan)
    return trace, seqs


def test_config4_schedule_matches_reference_engine(golden_meta):
    """Reduced config-4 workload: 95 steps with chunked prefill, two prefix-cache
    hits and a preemption with recompute."""
    g = golden_meta["e2e_config4_fp32"]
    w = e2e_config4_workload()
    trace, seqs = run_schedule(w["prompts"], w["max_new"], w["num_gpu_blocks"], w["max_num_batched_tokens"],
                               w["max_num_seqs"], w["min_chunk_size"], w["arrivals"], tokens=g["outputs"])
    assert g["preemptions"] >= 1
    ours = [{"rows": [[s.rid, "D" if c is None else "P", 0 if c is None else c, computed, table]
                      for s, c, computed, _, table in rows],
             "preempted": [s.rid for s in plan.preempted]} for plan, rows in trace]
    assert len(ours) == len(g["trace"]) == g["steps"]
    for i, (a, b) in enumerate(zip(ours, g["trace"])):
        assert a == b, f"step {i}: {a} != {b}"
    assert [s.out for s in seqs] == g["outputs"]
    assert any(s.preemptions for s in seqs)


def test_scripted_schedule_matches_reference_scheduler(golden_meta):
    """The scripted run behind the metadata fixtures: chunk floor 8, at most 6
    rows, a 64-token budget and shared prefixes (make_golden.scheduler_trace)."""
    shared = list(range(1000, 1040))
    prompts = [shared + list(range(7)), list(range(2000, 2070)), list(range(3000, 3016)), shared + [5, 6, 7]]
    sched = Scheduler(BlockPool(48), 64, 6, 8)
    seqs = [Seq(i, p, 3 + i) for i, p in enumerate(prompts)]
    arrivals = {0: [0, 1], 2: [2], 4: [3]}
    steps = []
    for step in range(40):
        for i in arrivals.get(step, []):
            sched.add(seqs[i])
        if not sched.has_unfinished():
            break
        plan = sched.plan()
        if not plan.rows:
            continue
        steps.append([{"phase": "NEEDS_DECODE" if c is None else "NEEDS_PREFILL", "chunk": 0 if c is None else c,
                       "num_computed_tokens": s.computed, "total_len": s.total_len, "block_table": list(s.table)}
                      for s, c in plan.rows])
        for s, c in plan.rows:
            if c is None or s.rid in plan.final:
                s.out.append(7)
        sched.commit(plan)
    ref = [st["rows"] for st in golden_meta["scheduler_trace"]]
    assert steps == ref
