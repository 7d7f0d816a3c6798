"""End to end through the registered "paged|b200" attention function: a seeded
tiny random Llama (fp32) served with continuous batching and chunked prefill
must emit exactly the greedy tokens the reference engine emitted on the same
weights and prompts (tests/golden: LLMEngine + Scheduler + BlockManager +
ModelRunner, eager paged attention, CPU). The smallest top-1/top-2 logit gap
along those tokens is 3.8e-3, far above fp32 noise."""
import numpy as np
import pytest
import torch

from serving_engine_b200 import check_device_errors
from serving_engine_b200.e2e import E2EEngine, config4_requests, random_llama
from tests.golden.cases import e2e_prompts

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("graphs", [False, True])
def test_greedy_tokens_match_reference_engine(golden_meta, graphs):
    """Also with the decode steps replayed from captured CUDA graphs."""
    g = golden_meta["e2e_tiny_fp32"]
    model = random_llama("tiny", seed=g["seed"], dtype=torch.float32, device="cuda")
    eng = E2EEngine(model, num_blocks=g["num_gpu_blocks"] + (1 if graphs else 0),
                    max_num_batched_tokens=g["max_num_batched_tokens"], use_graphs=graphs, max_context=256)
    if graphs:
        eng.capture_graphs()
    prompts, max_new = e2e_prompts()
    rids = [eng.add_request(p, max_new) for p in prompts]
    eng.run()
    check_device_errors()
    outs = {s.rid: s.out for s in eng.done}
    assert [outs[r] for r in rids] == g["outputs"]
    assert any(st.kind == "mixed" for st in eng.stats) or any(st.kind == "prefill" for st in eng.stats)
    if graphs:
        assert any(st.kind == "decode" for st in eng.stats)


def test_bf16_engine_runs_chunked_and_mixed_steps():
    """bf16 (tcgen05 prefill + tensor-core decode inside the model): every
    request finishes with the requested number of in-vocabulary tokens, and
    the schedule exercised chunked prefill and mixed prefill/decode steps."""
    model = random_llama("tiny", seed=1, dtype=torch.bfloat16, device="cuda")
    eng = E2EEngine(model, num_blocks=256, max_num_batched_tokens=96, max_num_seqs=8)
    prompts = config4_requests(seed=3, n=12, vocab=1000)
    prompts = [p[: 40 + 13 * i] for i, p in enumerate(prompts)]
    for p in prompts:
        eng.add_request(p, 9)
    eng.run()
    check_device_errors()
    assert len(eng.done) == 12 and all(len(s.out) == 9 for s in eng.done)
    assert all(0 <= t < 1000 for s in eng.done for t in s.out)
    assert {st.kind for st in eng.stats} >= {"mixed", "decode"}
    assert len(eng.free) == 256
