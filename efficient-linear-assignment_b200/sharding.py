"""Batch sharding of independent assignment problems across GPUs.

Problems of a batch share nothing (the reference's election and top-2 are per
problem and per row, torch_backend.py:93), so a batch splits into contiguous
slices, one per GPU, and every GPU solves its slice with no communication on
the solve path.  Two ways to drive it:

* one process per GPU (torchrun): ``shard_range`` picks this rank's slice and
  ``gather_assignments`` collects the (B_r, N) results on every rank
  (one all-gather of int64 indices after the solve, outside the solve);
* one process, several devices: ``solve_multi_device`` scatters the batch,
  launches every slice on its device's current stream without waiting, and
  gathers the results onto the input's device (device status checked after
  the gather).
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist


def shard_range(B: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) slice of B problems for `rank` of `world`.

    The first B % world ranks get one problem more.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(B, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_assignments(local: torch.Tensor, B: int, group=None) -> torch.Tensor:
    """All-gather every rank's (B_r, N) assignment slice into the full (B, N)."""
    world = dist.get_world_size(group)
    N = local.shape[1]
    sizes = [shard_range(B, world, r) for r in range(world)]
    width = max(b - a for a, b in sizes)
    pad = torch.full((width, N), -2, dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[: b - a] for p, (a, b) in zip(parts, sizes)], dim=0)


def solve_multi_device(cost: torch.Tensor, devices: Sequence[torch.device],
                       solve_fn: Callable[[torch.Tensor], tuple] | None = None, *,
                       epsilon=1e-2, max_iter: int = 1000):
    """Solve a (B,N,M) batch split over `devices` from one process.

    Default: every slice is copied to its device and its solve enqueued there
    without waiting (no status read between devices), so the GPUs run at the
    same time; the device status words are checked once, after the gather,
    and a device-side error raises AuctionError.  ``solve_fn(cost_slice)`` ->
    (assignment, prices[, status]) replaces the solve (it should not
    synchronise if the devices are to overlap).  Returns the full
    (assignment, prices) on cost's device.
    """
    B = cost.shape[0]
    outs = []
    for r, dev in enumerate(devices):
        a, b = shard_range(B, len(devices), r)
        if a == b:
            continue
        part = cost[a:b].to(dev, non_blocking=True)
        if solve_fn is None:
            from .solver import solve
            outs.append(solve(part, epsilon, max_iter, check=False, return_status=True))
        else:
            outs.append(solve_fn(part))
    assign = torch.cat([o[0].to(cost.device) for o in outs], dim=0)
    prices = torch.cat([o[1].to(cost.device) for o in outs], dim=0)
    from . import _lib
    for o in outs:
        if len(o) > 2 and isinstance(o[-1], torch.Tensor) and o[-1].dtype == torch.int32:
            _lib.check(int(o[-1].item()), f"auction kernel on {o[-1].device}")
    return assign, prices
