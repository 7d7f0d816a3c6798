"""Failure detection on the GPU without a fault: a bounded wait that nothing
completes gives up, reports SEB_ERRBIT_TIMEOUT through the error word, and the
CUDA context stays usable for the next (correct) call."""
import time

import pytest
import torch

from serving_engine_b200 import check_device_errors, ops, workloads
from tests.test_paged_decode_gpu import assert_close, run_b200, run_oracle

pytestmark = pytest.mark.gpu


def _timed_selftest(polls):
    check_device_errors()  # start from a clean error word
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ops.selftest_bounded_wait(polls)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    with pytest.raises(RuntimeError, match="timed out"):
        check_device_errors()
    return waited


def test_bounded_wait_gives_up_and_reports_timeout():
    short = _timed_selftest(64)
    longer = _timed_selftest(1024)
    print(f"unsatisfied mbarrier try_wait: about {longer / 1024 * 1e6:.2f} us per poll "
          f"(64 polls {short * 1e3:.2f} ms including the first launch, 1024 polls {longer * 1e3:.2f} ms)")
    assert longer < 60, longer
    # the context is intact: the next call runs and matches the oracle
    b = workloads.decode_batch(4, 1, 900, 32, 8, 128, torch.bfloat16, seed=77, num_blocks=300)
    o, lse = run_b200(b)
    o_ref, lse_ref = run_oracle(b)
    assert_close(o, lse, o_ref, lse_ref, torch.bfloat16)
