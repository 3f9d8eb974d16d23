"""Golden parity cases: seeded inputs, epsilon schedule and max_iter.

Used by make_golden.py (which runs the reference to record the expected
outputs) and by the tests (which regenerate the same inputs from the seeds).
"""
from __future__ import annotations

import torch

import efficient_linear_assignment_b200 as ela

W = ela.workloads


def _randint(shape, hi, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, hi, shape, generator=g).to(dtype)


def _diag_batch(seed=7):
    C = W.uniform(4, 32, 32, seed)
    C[0] = 100.0
    C[0].diagonal().zero_()
    return C


def _randn64(seed=5):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(2, 64, 64, generator=g, dtype=torch.float64)


# name -> (input factory, epsilon or schedule, max_iter)
CASES = {
    "cfg1": (lambda: W.cfg1(), 1e-2, 1000),
    "cfg2_fixed": (lambda: W.cfg2(), 1e-2, 1000),
    "cfg2_escale": (lambda: W.cfg2(), W.CFG2_SCHEDULE, 1000),
    "cfg2_maxiter10": (lambda: W.cfg2(), 1e-2, 10),
    "cfg3_f16": (lambda: W.cfg3(torch.float16), 1e-2, 1000),
    "cfg3_bf16": (lambda: W.cfg3(torch.bfloat16), 1e-2, 1000),
    "cfg4_head16": (lambda: W.cfg4()[:16].contiguous(), 1e-2, 1000),
    "cfg5_small": (lambda: W.cfg5(2, 512), 1.0 / 513, 1000),
    "cfg5_small_escale": (lambda: W.cfg5(2, 512), W.eps_schedule(16.0, 1.0 / 513, 0.25), 1000),
    "zeros": (lambda: torch.zeros(2, 32, 32), 1e-2, 1000),
    "flat": (lambda: torch.full((2, 32, 32), 10.0), 1e-2, 1000),
    "diag_batch": (_diag_batch, 1e-2, 2000),
    "fp64": (_randn64, 1e-3, 200),
    "rect_8x16": (lambda: W.uniform(2, 8, 16, 11), 1e-3, 2000),
    "rect_64x128": (lambda: W.uniform(2, 64, 128, 12), 1e-3, 2000),
    "wide_rows_16x8": (lambda: W.uniform(1, 16, 8, 13), 1e-2, 50),
    "robust_136": (lambda: W.uniform(2, 136, 136, 14), 1e-3, 5000),
}
for _n in (8, 16, 24, 40, 64, 96, 120):
    CASES[f"uniform_{_n}"] = (lambda n=_n: W.uniform(3, n, n, 20 + n), 1e-3, 2000)
for _n in (8, 24, 64, 120, 128, 200):
    CASES[f"ties_{_n}"] = (lambda n=_n: _randint((3, n, n), 4, 40 + n), 1.0 / (_n + 1), 3000)
