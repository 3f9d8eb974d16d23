"""GPU tests of the auction on implicit low-rank costs C = Q K^T
(ela_auction_solve_implicit: cost tiles on the tcgen05 tensor cores every round,
never stored).

Contract: every cost value is the fp32 result of one fixed MMA instruction
sequence, so the implicit solve must equal, bit for bit, the CPU oracle run on
the matrix the same instructions write out (ela_auction_implicit_costs); that
matrix must equal torch's fp32 product of the bf16/fp16 factors up to fp32
rounding of the dot products."""
import numpy as np
import pytest
import scipy.optimize
import torch

import efficient_linear_assignment_b200 as ela
from efficient_linear_assignment_b200 import _lib

pytestmark = pytest.mark.gpu


def _factors(B, N, M, D, dtype, seed, integer=False):
    g = torch.Generator().manual_seed(seed)
    if integer:  # small integers: exact products, many tied costs
        Q = torch.randint(-2, 3, (B, N, D), generator=g).float()
        K = torch.randint(-2, 3, (B, M, D), generator=g).float()
    else:
        Q = torch.randn(B, N, D, generator=g)
        K = torch.randn(B, M, D, generator=g)
    return Q.to(dtype), K.to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_implicit_costs_equal_fp32_product(dtype):
    for B, N, M, D in ((2, 128, 128, 16), (1, 300, 512, 64), (3, 64, 256, 128)):
        Q, K = _factors(B, N, M, D, dtype, seed=N + D)
        C = ela.implicit_costs(Q.cuda(), K.cuda()).cpu()
        ref = Q.double() @ K.double().transpose(1, 2)
        tol = 1e-6 * (Q.double().abs() @ K.double().abs().transpose(1, 2)) + 1e-30
        assert ((C.double() - ref).abs() <= tol).all()


CASES = [((4, 128, 128, 16), torch.bfloat16, False, 1e-2),
         ((2, 256, 512, 64), torch.bfloat16, False, [1.0, 0.1, 1e-2]),
         ((3, 512, 512, 16), torch.bfloat16, False, 1e-2),
         ((2, 100, 384, 32), torch.float16, False, 1e-2),
         ((2, 128, 128, 32), torch.bfloat16, True, 1.0 / 129),
         ((1, 300, 256, 16), torch.bfloat16, True, [4.0, 1.0 / 257])]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_implicit_solve_equals_oracle_on_its_costs(case, oracle_mod):
    (B, N, M, D), dtype, integer, eps = CASES[case]
    Q, K = _factors(B, N, M, D, dtype, seed=case, integer=integer)
    Qd, Kd = Q.cuda(), K.cuda()
    C = ela.implicit_costs(Qd, Kd).cpu()
    a, p, st = ela.solve_implicit(Qd, Kd, eps, 3000)
    ao, po, so = oracle_mod.solve(C, eps, 3000, nthreads=4)
    assert torch.equal(a.cpu(), ao) and torch.equal(p.cpu(), po)
    assert torch.equal(st[:, :2].cpu(), so[:, :2])


def test_implicit_solve_lowest_row_rule(oracle_mod):
    Q, K = _factors(2, 128, 128, 16, torch.bfloat16, seed=9, integer=True)
    C = ela.implicit_costs(Q.cuda(), K.cuda()).cpu()
    a, p, _ = ela.solve_implicit(Q.cuda(), K.cuda(), 1.0 / 129, 3000, tie_rule=ela.TIE_LOWEST_ROW)
    ao, po, _ = oracle_mod.solve(C, 1.0 / 129, 3000, tie_rule=1)
    assert torch.equal(a.cpu(), ao) and torch.equal(p.cpu(), po)


def test_implicit_solve_within_bound_of_scipy():
    B, N, M, D = 2, 256, 256, 64
    Q, K = _factors(B, N, M, D, torch.bfloat16, seed=3)
    a, _, st = ela.solve_implicit(Q.cuda(), K.cuda(), [1.0, 0.1, 1e-3], 5000)
    C = (Q.double() @ K.double().transpose(1, 2)).numpy()
    for b in range(B):
        an = a[b].cpu().numpy()
        assert (an >= 0).all() and len(np.unique(an)) == N
        r, c = scipy.optimize.linear_sum_assignment(C[b])
        assert C[b][np.arange(N), an].sum() - C[b][r, c].sum() <= N * 1e-3 + 1e-3


def test_implicit_rejects_unsupported_shapes():
    Q = torch.zeros(1, 64, 24, dtype=torch.bfloat16, device="cuda")  # D not a multiple of 16
    K = torch.zeros(1, 128, 24, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ela.AuctionError) as ei:
        ela.solve_implicit(Q, K)
    assert ei.value.status == _lib.ELA_ERR_ARGUMENT
