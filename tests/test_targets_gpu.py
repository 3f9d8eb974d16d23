"""GPU checks at the benchmark configurations' full sizes and of the options
beside the reference's own mode.

* Every solve is a valid permutation whose total cost is within N * eps_final
  of scipy's exact ``linear_sum_assignment`` optimum (the reference's own
  bound test is tests/test_robustness.py:49-60, at 1.5 * N * eps).
* Config 5's convergent mode (epsilon scaled from the cost range 16 down to
  1/(N+1)) returns the exact optimum of an 8192 x 8192 integer problem.
* ``tie_rule=TIE_LOWEST_ROW`` equals the CPU oracle run with the same rule and
  keeps the bound.
* ``auto_pad`` on tie-heavy integer costs equals the oracle run on the
  explicitly padded tensor (``pad_input``), unpadded.
"""
import numpy as np
import pytest
import scipy.optimize
import torch

import efficient_linear_assignment_b200 as ela

pytestmark = pytest.mark.gpu


def _check_bound(cost_cpu, assign, eps_final):
    """Valid permutation per problem, total within N * eps_final of optimal."""
    B, N, M = cost_cpu.shape
    c64 = cost_cpu.double().numpy()
    for b in range(B):
        a = assign[b].cpu().numpy()
        assert (a >= 0).all(), "unassigned rows left"
        assert len(np.unique(a)) == N, "two rows share a column"
        r, c = scipy.optimize.linear_sum_assignment(c64[b])
        opt = c64[b][r, c].sum()
        mine = c64[b][np.arange(N), a].sum()
        assert mine - opt <= N * eps_final + 1e-6 * abs(opt), (mine, opt)


@pytest.mark.parametrize("case", ["cfg2_escale", "cfg2_fixed", "cfg3_f16", "cfg3_bf16"])
def test_full_size_within_bound_of_scipy(case):
    if case.startswith("cfg2"):
        cost = ela.workloads.cfg2()
        eps = ela.workloads.CFG2_SCHEDULE if case == "cfg2_escale" else [1e-2]
    else:
        cost = ela.workloads.cfg3(torch.float16 if case == "cfg3_f16" else torch.bfloat16)
        eps = [1e-2]
    a, _, st = ela.solve(cost.cuda(), eps, 1000)
    assert int(st[0, 3]) == 0
    _check_bound(cost.float(), a, eps[-1])


def test_cfg5_convergent_mode_is_exact_at_8192():
    cost = ela.workloads.cfg5(8, 8192)[5:6].contiguous()
    N = cost.shape[1]
    sched = ela.workloads.eps_schedule(16.0, 1.0 / (N + 1), 0.25)
    a, _, st = ela.solve(cost.cuda(), sched, 20000)
    assert int(st[0, 3]) == 0
    c = cost[0].float().numpy()
    r, cc = scipy.optimize.linear_sum_assignment(c)
    an = a[0].cpu().numpy()
    assert len(np.unique(an)) == N
    assert c[np.arange(N), an].sum() == c[r, cc].sum()  # integer costs, eps < 1/N: optimal


@pytest.mark.parametrize("path", [ela.PATH_CTA, ela.PATH_GRID, ela.PATH_CLUSTER])
def test_lowest_row_rule_matches_oracle_and_bound(path, oracle_mod):
    g = torch.Generator().manual_seed(31)
    cases = [
        (torch.rand(2, 256, 256, generator=g), 1e-3),
        ((torch.rand(3, 136, 136, generator=g) * 6).floor(), 1.0 / 137),  # integer costs: ties
        (ela.workloads.cfg5(2, 512), ela.workloads.eps_schedule(16.0, 1.0 / 513, 0.25)),  # convergent mode
    ]
    for cost, eps in cases:
        a, p, st = ela.solve(cost.cuda(), eps, 20000, path=path, tie_rule=ela.TIE_LOWEST_ROW)
        ao, po, so = oracle_mod.solve(cost, eps, 20000, nthreads=4, tie_rule=1)
        assert torch.equal(a.cpu(), ao) and torch.equal(p.cpu(), po)
        assert torch.equal(st[:, :2].cpu(), so[:, :2])
        eps_final = eps[-1] if isinstance(eps, list) else eps
        _check_bound(cost.float(), a, eps_final)


def test_lowest_row_rule_differs_from_reference_somewhere(oracle_mod):
    """The option changes the election (else it would be untested)."""
    cost = (torch.rand(1, 256, 256, generator=torch.Generator().manual_seed(5)) * 4).floor()
    hi, _, _ = ela.solve(cost.cuda(), 1.0 / 257, 5000)
    lo, _, _ = ela.solve(cost.cuda(), 1.0 / 257, 5000, tie_rule=ela.TIE_LOWEST_ROW)
    assert not torch.equal(hi, lo)


@pytest.mark.parametrize("shape", [(1, 16, 21), (1, 120, 121), (2, 13, 16), (2, 130, 133), (1, 133, 130),
                                   (3, 7, 9)])
def test_auto_pad_tie_heavy_equals_oracle_on_padded_tensor(shape, oracle_mod):
    """Integer costs (many tied maxima): auto_pad returns the real rows of the
    oracle's solve of pad_input(cost), whichever branch auto_pad takes."""
    B, N, M = shape
    g = torch.Generator().manual_seed(N * 1000 + M)
    cost = torch.randint(0, 5, (B, N, M), generator=g).float()
    padded, orig = ela.pad_input(cost)
    ao, _, _ = oracle_mod.solve(padded, 1e-2, 3000)
    expect = ela.unpad_result(ao.clamp(min=0), orig)
    got = ela.linear_assignment(cost.cuda(), epsilon=1e-2, max_iter=3000, auto_pad=True)
    assert torch.equal(got.cpu(), expect)
