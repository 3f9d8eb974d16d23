"""Sharded solves on two or more GPUs: one process per GPU over NCCL (as
``bench.py --gpus N`` runs them), every rank solving its contiguous slice of
the batch with no communication on the solve path, then one all-gather of the
indices.  The gathered batch must equal the CPU oracle's solve of the whole
batch, bit for bit (problems are independent, so sharding changes nothing).
Skipped on a one-GPU machine."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two or more GPUs")]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    import efficient_linear_assignment_b200 as ela
    from efficient_linear_assignment_b200.sharding import gather_assignments, shard_range
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        results = {}
        # cfg4-like batch (one-CTA path) and a few 2048^2 problems (cluster path)
        for name, cost, eps in (("cfg4_slice", ela.workloads.cfg4()[:24].contiguous(), [1e-2]),
                                ("large", ela.workloads.uniform(3, 2048, 2048, seed=9), [1.0, 0.1, 1e-2])):
            a, b = shard_range(cost.shape[0], world, rank)
            local, _, _ = ela.solve(cost[a:b].cuda(), eps, 1000)
            results[name] = gather_assignments(local, cost.shape[0]).cpu()
        q.put((rank, results))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_nccl_sharded_batches_equal_oracle(oracle_mod):
    import efficient_linear_assignment_b200 as ela
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    expect = {"cfg4_slice": oracle_mod.solve(ela.workloads.cfg4()[:24].contiguous(), 1e-2, 1000, nthreads=8)[0],
              "large": oracle_mod.solve(ela.workloads.uniform(3, 2048, 2048, seed=9), [1.0, 0.1, 1e-2], 1000,
                                        nthreads=8)[0]}
    for _, results in res:
        for name, full in results.items():
            assert torch.equal(full, expect[name]), name
