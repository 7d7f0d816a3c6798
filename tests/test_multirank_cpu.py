"""Host-side logic of the multi-GPU bench path, run as world_size-2 gloo ranks
on CPU: kv-head sharding of the decode workload and max-over-ranks timing."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        spec = bench.shard_spec(64, world, rank, seed=0)
        slowest = bench.max_over_ranks(dist, 10.0 + rank, torch.device("cpu"))
        q.put((rank, spec, slowest))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_shard_spec_and_max_over_ranks_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert [r[2] for r in results] == [10.0 + world - 1] * world  # every rank sees the slowest time
    specs = [r[1] for r in results]
    assert all(s["batch"] == 64 * world and s["hkv"] == 8 // world and s["hq"] == 32 // world for s in specs)
    assert len({s["seed"] for s in specs}) == world  # ranks hold different data
    # per-rank units equal the 1-GPU config: batch x kv heads
    assert specs[0]["batch"] * specs[0]["hkv"] == 64 * 8


def test_shard_spec_rejects_indivisible_heads():
    with pytest.raises(ValueError):
        bench.shard_spec(64, 3, 0, seed=0)


def _tp_mlp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from serving_engine_b200.tp_decode import TPConfig, TPLlamaDecoder

        cfg = TPConfig(layers=1, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=50)
        dec = TPLlamaDecoder(cfg, rank, world, torch.device("cpu"), batch=3, context=20, seed=5, fill_kv=False)
        h = torch.randn(3, 64, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
        out = dec.mlp(h, dec.layers[0]).float()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_tp_mlp_shards_sum_to_full_mlp_gloo():
    """Column-parallel gate/up + row-parallel down + all-reduce over 2 gloo ranks
    equals the unsharded SwiGLU of the same seeded weights."""
    from serving_engine_b200.tp_decode import TPConfig, TPLlamaDecoder

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_mlp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cfg = TPConfig(layers=1, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=50)
    full = TPLlamaDecoder(cfg, 0, 1, torch.device("cpu"), batch=3, context=20, seed=5, fill_kv=False)
    h = torch.randn(3, 64, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
    ref = full.mlp(h, full.layers[0]).float()
    torch.testing.assert_close(outs[0], ref, atol=2e-3, rtol=2e-2)
    torch.testing.assert_close(outs[0], outs[1], atol=0, rtol=0)  # every rank holds the reduced sum


def _leaving_worker(rank, world, port, q):
    """Rank 1 leaves between steps (exits without joining the next collective);
    rank 0 must learn of it through its process group's short timeout, as an
    error from the collective rather than a hang."""
    import datetime
    import time

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # a slow-starting rank must not fail the rendezvous: only the collectives'
    # group carries the short timeout
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    group = dist.new_group(list(range(world)), timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t, group=group)  # one step together
    if rank == 1:
        q.put((rank, "left", float(t[0])))
        q.close()
        q.join_thread()  # the message is out before the process goes
        os._exit(0)  # leave without the next collective or a clean shutdown
    t0 = time.monotonic()
    try:
        dist.all_reduce(t, group=group)
        q.put((rank, "no error", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - the backend's error type varies
        q.put((rank, f"error: {type(e).__name__}", time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_leaving_ends_peer_collective_with_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict((r, (msg, v)) for r, msg, v in (q.get(timeout=300) for _ in procs))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert outs[1][0] == "left" and outs[1][1] == 2.0
    msg, waited = outs[0]
    assert msg.startswith("error"), msg
    assert waited < 60, waited
