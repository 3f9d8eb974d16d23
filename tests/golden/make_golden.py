"""Record golden outputs by running the REFERENCE solver (not this project).

Point ELA_REFERENCE_SRC at the reference project's `src` directory (the one
that holds the `efficient_linear_assignment` package) and run:

    ELA_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_golden.py

For every case of cases.py it runs the reference's AuctionTorch.solve
(src/efficient_linear_assignment/auction/torch_backend.py:9-159) on one CPU
thread (its only well-defined setting) and writes golden_<case>.npz with the
assignment, the prices and a SHA-256 of the input bytes.  Half inputs are
solved as cost.float() (fp32 prices).  Epsilon schedules call the reference
once per epsilon with the previous prices as the starting prices: the
reference hard-codes zero starting prices (torch_backend.py:27), so its
module-level `torch` is swapped for a proxy whose `zeros` returns the warm
prices for that one call; the reference code itself runs unmodified.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
if not os.environ.get("ELA_REFERENCE_SRC"):
    sys.exit("set ELA_REFERENCE_SRC to the reference project's src directory")
sys.path.insert(0, os.environ["ELA_REFERENCE_SRC"])
sys.dont_write_bytecode = True

from efficient_linear_assignment.auction import torch_backend as ref_tb  # noqa: E402

sys.path.insert(0, HERE)
from cases import CASES  # noqa: E402
from make_golden_io import input_digest  # noqa: E402


class _WarmTorch:
    """Delegates to torch; `zeros` returns the given warm prices once."""

    def __init__(self, warm):
        self._warm = warm

    def __getattr__(self, name):
        return getattr(torch, name)

    def zeros(self, *a, **k):
        if self._warm is not None:
            w, self._warm = self._warm, None
            return w.clone()
        return torch.zeros(*a, **k)


def reference_solve(cost, eps, max_iter):
    if cost.dtype in (torch.float16, torch.bfloat16):
        cost = cost.float()
    sched = [eps] if isinstance(eps, (int, float)) else list(eps)
    prices = None
    for e in sched:
        saved = ref_tb.torch
        ref_tb.torch = _WarmTorch(prices)
        try:
            assign, prices = ref_tb.AuctionTorch(e, max_iter).solve(cost)
        finally:
            ref_tb.torch = saved
    return assign, prices


def main(names=None):
    torch.set_num_threads(1)
    for name, (make, eps, max_iter) in CASES.items():
        if names and name not in names:
            continue
        cost = make()
        a, p = reference_solve(cost, eps, max_iter)
        out = os.path.join(HERE, f"golden_{name}.npz")
        np.savez_compressed(out, assign=a.numpy().astype(np.int32), prices=p.numpy(),
                            digest=np.array(input_digest(cost)))
        print(f"{name}: unassigned={(a == -1).sum().item()} -> {os.path.basename(out)}")


if __name__ == "__main__":
    main(sys.argv[1:])
