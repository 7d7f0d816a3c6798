"""Failure detection on the GPU without a fault: a bounded wait that nothing
completes gives up, reports SEB_ERRBIT_TIMEOUT through the error word, and the
CUDA context stays usable for the next (correct) call."""
import time

import pytest
import torch

from serving_engine_b200 import check_device_errors, ops, workloads
from tests.test_paged_decode_gpu import assert_close, run_b200, run_oracle

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports_timeout():
    check_device_errors()  # start from a clean error word
    t0 = time.perf_counter()
    ops.selftest_bounded_wait(4096)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    with pytest.raises(RuntimeError, match="timed out"):
        check_device_errors()
    assert waited < 30, waited
    # the context is intact: the next call runs and matches the oracle
    b = workloads.decode_batch(4, 1, 900, 32, 8, 128, torch.bfloat16, seed=77, num_blocks=300)
    o, lse = run_b200(b)
    o_ref, lse_ref = run_oracle(b)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)
