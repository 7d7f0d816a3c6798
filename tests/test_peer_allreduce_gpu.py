"""All-reduce fused with residual add + RMSNorm (seb_allreduce_add_rmsnorm).

On one GPU the ranks' peer regions sit on the same device and one cooperative
launch runs every rank's part, so the flag protocol, the row ownership and the
pushes to every rank are exercised exactly as across GPUs. Every rank's
residual must equal x + S bit for bit (S: the ranks' partials summed in fp32 in
rank order and rounded once), every rank's output must be bit-identical to
seb_add_rmsnorm applied to that sum, and within one rounding of an fp32 RMSNorm.
With two GPUs, the two-process run must match NCCL all-reduce followed by
seb_add_rmsnorm bit for bit (a two-operand sum rounds the same either way).
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from serving_engine_b200 import check_device_errors, ops
from serving_engine_b200.peer_allreduce import PeerAllReduceNorm
from tests.test_layer_ops_gpu import assert_within_ulp

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def reduced(partials):
    s = partials[0].float()
    for p in partials[1:]:
        s = s + p.float()
    return s.to(partials[0].dtype)


def fill(ar, world, gen, x0):
    parts = []
    for q in range(world):
        p, x, _ = ar.views(q)
        p.copy_(torch.randn(p.shape, generator=gen, device=DEV).to(p.dtype))
        x.copy_(x0)
        parts.append(p.clone())
    return parts


def check_call(ar, world, parts, x0, w, eps=1e-5):
    s = reduced(parts)
    x_ref = x0.clone()
    out_ref = ops.add_rmsnorm(x_ref, s, w, eps)  # x_ref <- x0 + s, out_ref = rmsnorm
    xf = x_ref.float()
    for q in range(world):
        _, x, out = ar.views(q)
        assert torch.equal(x, x_ref), f"rank {q} residual"
        assert torch.equal(out, out_ref), f"rank {q} output"
        assert_within_ulp(out, xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("world,n,hidden", [(2, 256, 4096), (4, 6, 512), (8, 256, 4096), (3, 1, 2048),
                                            (2, 37, 10000), (1, 5, 4096)])
def test_single_device_ranks(dtype, world, n, hidden):
    gen = torch.Generator(device=DEV).manual_seed(world * 1000 + n)
    ar = PeerAllReduceNorm.single_device(world, n, hidden, dtype, DEV)
    try:
        w = (1 + 0.1 * torch.randn(hidden, generator=gen, device=DEV)).to(dtype)
        x0 = torch.randn(n, hidden, generator=gen, device=DEV).to(dtype)
        for _ in range(3):  # successive calls: the flag epochs advance
            parts = fill(ar, world, gen, x0)
            ar(w, 1e-5)
            torch.cuda.synchronize()
            check_device_errors(DEV)
            check_call(ar, world, parts, x0, w)
    finally:
        ar.close()


def test_single_device_graph_replay():
    world, n, hidden, dtype = 4, 64, 4096, torch.bfloat16
    gen = torch.Generator(device=DEV).manual_seed(5)
    ar = PeerAllReduceNorm.single_device(world, n, hidden, dtype, DEV)
    try:
        w = (1 + 0.1 * torch.randn(hidden, generator=gen, device=DEV)).to(dtype)
        x0 = torch.randn(n, hidden, generator=gen, device=DEV).to(dtype)
        fill(ar, world, gen, x0)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ar(w, 1e-5)  # warm-up outside the graph
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ar(w, 1e-5)
        for _ in range(3):
            parts = fill(ar, world, gen, x0)
            g.replay()
            torch.cuda.synchronize()
            check_device_errors(DEV)
            check_call(ar, world, parts, x0, w)
        del g
    finally:
        ar.close()


def test_missing_peer_times_out_and_context_survives():
    """Rank 0 runs alone; rank 1's flags are never set: every wait gives up after
    its bound, the error word says so, and the device keeps working."""
    world, n, hidden = 2, 8, 512
    ar = PeerAllReduceNorm.single_device(world, n, hidden, torch.bfloat16, DEV)
    try:
        w = torch.ones(hidden, dtype=torch.bfloat16, device=DEV)
        ar._launch(w, 1e-5, rank=0, all_ranks=False, polls=2000)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="timed out"):
            check_device_errors(DEV)
        y = torch.ones(4, device=DEV) * 2
        assert float(y.sum()) == 8.0
    finally:
        ar.close()


def test_rejects_bad_arguments():
    with pytest.raises(ValueError):
        PeerAllReduceNorm.single_device(9, 4, 512, torch.bfloat16, DEV)
    with pytest.raises(ValueError):
        PeerAllReduceNorm.single_device(2, 4, 500, torch.bfloat16, DEV)
    ar = PeerAllReduceNorm.single_device(2, 4, 512, torch.bfloat16, DEV)
    try:
        with pytest.raises(ValueError):
            ar(torch.ones(256, dtype=torch.bfloat16, device=DEV), 1e-5)
    finally:
        ar.close()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        n, hidden = 256, 4096
        ar = PeerAllReduceNorm(n, hidden, torch.bfloat16, dev)
        gen = torch.Generator(device=dev).manual_seed(0)
        w = (1 + 0.1 * torch.randn(hidden, generator=gen, device=dev)).bfloat16()
        x0 = torch.randn(n, hidden, generator=gen, device=dev).bfloat16()  # same on every rank
        ok = True
        for step in range(3):
            g = torch.Generator(device=dev).manual_seed(100 * step + rank)
            part = torch.randn(n, hidden, generator=g, device=dev).bfloat16()
            ar.partial.copy_(part)
            ar.x.copy_(x0)
            ar(w, 1e-5)
            nccl_sum = part.clone()
            dist.all_reduce(nccl_sum)
            x_ref = x0.clone()
            out_ref = ops.add_rmsnorm(x_ref, nccl_sum, w, 1e-5)
            torch.cuda.synchronize()
            check_device_errors(dev)
            ok &= bool(torch.equal(ar.x, x_ref)) and bool(torch.equal(ar.out, out_ref))
        q.put((rank, ok))
        ar.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_processes_match_nccl_then_norm():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res == {0: True, 1: True}
