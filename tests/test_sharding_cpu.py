"""CPU tests of the batch-sharding host logic (world_size 2 over gloo)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from efficient_linear_assignment_b200.sharding import gather_assignments, shard_range, solve_multi_device


@pytest.mark.parametrize("B,world", [(256, 8), (8, 3), (1, 2), (5, 8), (0, 2)])
def test_shard_ranges_partition_the_batch(B, world):
    covered = []
    for r in range(world):
        a, b = shard_range(B, world, r)
        assert 0 <= a <= b <= B
        covered += list(range(a, b))
    assert covered == list(range(B))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, B, N, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a, b = shard_range(B, world, rank)
    local = torch.arange(a * N, b * N, dtype=torch.int64).view(b - a, N)  # stands in for a solve
    full = gather_assignments(local, B)
    q.put((rank, full))
    dist.barrier()
    dist.destroy_process_group()


def test_gather_assignments_gloo_world2():
    B, N, world = 5, 4, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    expect = torch.arange(B * N, dtype=torch.int64).view(B, N)
    for _, full in res:
        assert torch.equal(full, expect)


def test_solve_multi_device_reassembles_in_order():
    cost = torch.rand(7, 8, 8)
    seen = []

    def fake_solve(part):
        seen.append(part.shape[0])
        return part.argmin(dim=2), part.amin(dim=1)

    a, p = solve_multi_device(cost, [torch.device("cpu")] * 3, fake_solve)
    assert seen == [3, 2, 2]
    assert torch.equal(a, cost.argmin(dim=2)) and torch.equal(p, cost.amin(dim=1))
