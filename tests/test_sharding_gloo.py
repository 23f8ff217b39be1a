"""Host-side sharding logic on CPU with two gloo ranks: each rank multiplies A by its column
shard of B, the shards are all-gathered and unsharded, and the result must equal the full
product on every rank."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import sharding


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        A = torch.randint(-3, 4, (M, K), generator=g).double()
        B = torch.randint(-3, 4, (K, N), generator=g).double()
        C_local = A @ sharding.local_shard(B, world, rank)
        C = sharding.gather_columns(C_local, world)
        q.put((rank, bool(torch.equal(C, A @ B))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gather_columns_matches_full_product(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 24, 40, 16, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in range(world))
    assert all(results.values()), results


def test_shard_bounds_and_unshard_cpu():
    assert sharding.shard_bounds(64, 4, 2) == (32, 48)
    with pytest.raises(ValueError):
        sharding.shard_bounds(10, 4, 0)
    M, N, world = 3, 8, 4
    full = torch.arange(M * N).reshape(M, N).float()
    shardmajor = torch.stack([full[:, r * 2:(r + 1) * 2] for r in range(world)])
    assert torch.equal(sharding.unshard(shardmajor, M, N, world), full)


def _failing_worker(rank, world, port, q):
    """Rank 1 leaves before the gather (an exception on the host, between steps); rank 0's
    gather must end with an error within the process group's timeout instead of hanging."""
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()
        os._exit(0)  # no destroy_process_group, no gather: the peer simply disappears
    t0 = time.time()
    try:
        sharding.gather_columns(torch.ones(4, 8), world)
        q.put((rank, "no error"))
    except Exception as e:  # gloo reports the lost peer (timeout or connection closed)
        q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_gather_reports_a_lost_rank_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results = {}
    for _ in range(2):
        r, msg = q.get(timeout=10)
        results[r] = msg
    assert results[1] == "left"
    assert results[0].startswith("error after"), results
