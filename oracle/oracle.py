"""CPU oracle for the auction solver -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module, always as the checker.  The product path (the CUDA library behind
``efficient_linear_assignment_b200``) never imports it.

``solve`` wraps ``auction_oracle.c`` (a C restatement of the reference's
``AuctionTorch.solve``, src/efficient_linear_assignment/auction/torch_backend.py:9-159,
as run with one torch thread).  ``solve_numpy`` is an independent pure-numpy
restatement of the same rounds for small cases; the two are checked against
each other and against golden vectors produced by the reference itself
(tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libela_oracle.so")
_lib = None

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}


def build() -> str:
    """Compile the C oracle in place (oracle/libela_oracle.so)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        lib.ela_oracle_solve.restype = ctypes.c_int
        lib.ela_oracle_solve.argtypes = [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(ctypes.c_double), ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
        ]
        _lib = lib
    return _lib


def eps_schedule(eps0: float, eps_final: float, factor: float) -> list[float]:
    """Geometric epsilon schedule eps0, eps0*f, ... while > eps_final, then eps_final."""
    out, e = [], float(eps0)
    while e > eps_final:
        out.append(e)
        e *= factor
    out.append(float(eps_final))
    return out


def solve(cost: torch.Tensor, eps, max_iter: int = 1000, nthreads: int = 1, tie_rule: int = 0):
    """Oracle solve of a (B,N,M) CPU cost tensor.

    eps: a float (the reference's constant epsilon) or a list (epsilon schedule).
    tie_rule: 0 = the reference's election (highest row among the bids within
    1e-5 of the new price), 1 = lowest row (a variant, not the reference).
    Returns (assignment int64 (B,N) with -1 = unassigned, prices (B,M) float32 or
    float64, stats int64 (B,4) = [rounds, row_bids, tied_row_bids, unassigned]).
    """
    lib = _load()
    if cost.dim() == 2:
        cost = cost.unsqueeze(0)
    cost = cost.detach().cpu().contiguous()
    B, N, M = cost.shape
    sched = [float(eps)] if isinstance(eps, (int, float)) else [float(e) for e in eps]
    e_arr = (ctypes.c_double * len(sched))(*sched)
    assign = torch.empty((B, N), dtype=torch.int64)
    pdt = torch.float64 if cost.dtype == torch.float64 else torch.float32
    prices = torch.empty((B, M), dtype=pdt)
    stats = torch.zeros((B, 4), dtype=torch.int64)
    rc = lib.ela_oracle_solve(
        ctypes.c_void_p(cost.data_ptr()), DTYPE_CODE[cost.dtype], B, N, M, N * M, M,
        e_arr, len(sched), int(max_iter), int(tie_rule), ctypes.c_void_p(assign.data_ptr()),
        ctypes.c_void_p(prices.data_ptr()), ctypes.c_void_p(stats.data_ptr()), int(nthreads))
    if rc != 0:
        raise ValueError(f"oracle rejected arguments (status {rc})")
    return assign, prices, stats


def bids(cost: torch.Tensor, eps: float, prices: torch.Tensor | None = None,
         assignment: torch.Tensor | None = None):
    """Oracle of one round's bids (the checker of ela_auction_compute_bids):
    (B,N,M) CPU cost, optional (B,M) prices (float32, float64 for fp64 costs)
    and (B,N) int64 assignment (-1 = bids).  Returns (best_idx int64 (B,N),
    increments (B,N)): torch.topk's column on (-c) - P and (v1 - v2) + eps
    (torch_backend.py:65-88); -1 and 0 for assigned rows."""
    lib = _load()
    if not hasattr(lib, "_bids_ready"):
        lib.ela_oracle_bids.restype = ctypes.c_int
        lib.ela_oracle_bids.argtypes = [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_double, ctypes.c_void_p, ctypes.c_void_p]
        lib._bids_ready = True
    if cost.dim() == 2:
        cost = cost.unsqueeze(0)
    cost = cost.detach().cpu().contiguous()
    B, N, M = cost.shape
    pdt = torch.float64 if cost.dtype == torch.float64 else torch.float32
    P = None if prices is None else prices.detach().cpu().to(pdt).contiguous()
    A = None if assignment is None else assignment.detach().cpu().to(torch.int64).contiguous()
    idx = torch.empty((B, N), dtype=torch.int64)
    inc = torch.empty((B, N), dtype=pdt)
    rc = lib.ela_oracle_bids(ctypes.c_void_p(cost.data_ptr()), DTYPE_CODE[cost.dtype], B, N, M, N * M, M,
                             None if P is None else ctypes.c_void_p(P.data_ptr()),
                             None if A is None else ctypes.c_void_p(A.data_ptr()), float(eps),
                             ctypes.c_void_p(idx.data_ptr()), ctypes.c_void_p(inc.data_ptr()))
    if rc != 0:
        raise ValueError(f"oracle rejected arguments (status {rc})")
    return idx, inc


def solve_numpy(cost: np.ndarray, eps: float, max_iter: int = 1000):
    """Pure-numpy restatement of torch_backend.py:54-156 for one (N,M) problem.

    For small cases only.  Returns (assignment (N,) int64, prices (M,), tied flag).
    Column ties go to the lowest column (np.argmax), as in the C oracle.
    """
    R = np.float64 if cost.dtype == np.float64 else np.float32
    ben = (-cost.astype(R))
    N, M = ben.shape
    P = np.zeros(M, dtype=R)
    assign = np.full(N, -1, dtype=np.int64)
    owner = np.full(M, -1, dtype=np.int64)
    tied = False
    for _ in range(max_iter):
        act = np.nonzero(assign == -1)[0]
        if act.size == 0:
            break
        v = ben[act] - P[None, :]
        j1 = np.argmax(v, axis=1)
        v1 = v[np.arange(act.size), j1]
        v_masked = v.copy()
        v_masked[np.arange(act.size), j1] = -np.inf
        v2 = v_masked.max(axis=1)
        tied |= bool(np.any(v2 == v1))
        inc = (v1 - v2) + R(eps)
        bids = (P[j1] + inc).astype(R)
        np.maximum.at(P, j1, bids)
        win = np.abs(bids - P[j1]) < R(1e-5)
        elected = {}
        for k in np.nonzero(win)[0]:
            elected[int(j1[k])] = int(act[k])  # ascending rows: last writer wins
        for j, w in elected.items():
            prev = owner[j]
            if prev != -1:
                assign[prev] = -1
            owner[j] = w
            assign[w] = j
    return assign, P, tied
