"""CPU tests: the oracle against golden vectors recorded from the reference,
and its column tie rule against torch.topk."""
import numpy as np
import pytest
import torch

from cases import CASES
from make_golden_io import load_golden, input_digest


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name, oracle_mod):
    make, eps, max_iter = CASES[name]
    cost = make()
    g = load_golden(name)
    assert input_digest(cost) == g["digest"], "input generator drifted from the golden recording"
    a, p, st = oracle_mod.solve(cost, eps, max_iter, nthreads=4)
    assert np.array_equal(a.numpy(), g["assign"].astype(np.int64))
    assert np.array_equal(p.numpy(), g["prices"])


@pytest.mark.parametrize("M", [2, 3, 5, 8, 16, 40, 96, 120, 127, 128, 129, 256, 1000])
def test_topk_tie_rule_matches_torch(M, oracle_mod):
    """A one-row problem is won in round 1 by the column torch.topk(-cost) reports."""
    torch.set_num_threads(1)
    g = torch.Generator().manual_seed(M)
    for trial in range(200):
        hi = [2, 3, 6][trial % 3]
        cost = torch.randint(0, hi, (1, 1, M), generator=g).float()
        a, _, _ = oracle_mod.solve(cost, 0.5, 1)
        expect = torch.topk(-cost[0], 2, dim=1).indices[0, 0].item()
        assert a[0, 0].item() == expect, (trial, cost.flatten().tolist())


@pytest.mark.parametrize("n", [8, 24, 64])
def test_c_oracle_equals_numpy_restatement(n, oracle_mod):
    g = torch.Generator().manual_seed(100 + n)
    cost = torch.rand(2, n, n, generator=g)
    a, p, _ = oracle_mod.solve(cost, 1e-3, 500)
    for b in range(2):
        a2, p2, tied = oracle_mod.solve_numpy(cost[b].numpy(), 1e-3, 500)
        if not tied:
            assert np.array_equal(a[b].numpy(), a2)
            assert np.array_equal(p[b].numpy(), p2)


def test_oracle_threads_do_not_change_results(oracle_mod):
    cost = CASES["cfg4_head16"][0]()
    a1, p1, _ = oracle_mod.solve(cost, 1e-2, 1000, nthreads=1)
    a8, p8, _ = oracle_mod.solve(cost, 1e-2, 1000, nthreads=8)
    assert torch.equal(a1, a8) and torch.equal(p1, p8)


@pytest.mark.parametrize("shape", [(2, 13, 21), (1, 16, 21), (3, 7, 9), (2, 30, 45), (1, 17, 17)])
def test_direct_solve_equals_padded_solve_when_dummy_rows_fit(shape, oracle_mod):
    """The equivalence auto_pad relies on: with M padded and no more dummy rows
    than dummy columns, the real rows of solve(pad_input(C)) equal solve(C)."""
    import efficient_linear_assignment_b200 as ela
    B, N, M = shape
    pn, pm = ela.get_pad_size(N), ela.get_pad_size(M)
    assert pm > 0 and pn <= pm
    g = torch.Generator().manual_seed(N + 7 * M)
    cost = torch.rand(B, N, M, generator=g)
    padded, _ = ela.pad_input(cost)
    ap, _, _ = oracle_mod.solve(padded, 1e-3, 2000)
    ad, _, _ = oracle_mod.solve(cost, 1e-3, 2000)
    assert torch.equal(ap[:, :N], ad)


@pytest.mark.parametrize("M", [16, 96, 127, 128, 200])
def test_oracle_bids_match_torch_topk(M, oracle_mod):
    # one round's bids of the oracle against torch.topk itself (one thread, as
    # the reference runs), on tie-heavy integer rows with a few price levels
    torch.set_num_threads(1)
    g = torch.Generator().manual_seed(M)
    cost = torch.randint(0, 4, (2, 64, M), generator=g).float()
    prices = torch.randint(0, 3, (2, M), generator=g).float() * 0.5
    idx, inc = oracle_mod.bids(cost, 0.01, prices)
    v = (-cost) - prices[:, None, :]
    top = torch.topk(v, 2, dim=2)
    assert torch.equal(idx, top.indices[..., 0])
    assert torch.equal(inc, (top.values[..., 0] - top.values[..., 1]) + torch.tensor(0.01, dtype=torch.float32))
