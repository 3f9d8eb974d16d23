"""GPU tests of the bid pass alone (ela_auction_compute_bids, the reference's
compute_bids, src/csrc/interface.cpp:31-40): for every unassigned row, the
column torch.topk picks on -cost - prices and the increment (v1 - v2) + eps
must equal the CPU oracle's one round (torch_backend.py:65-88) bit for bit,
ties included; assigned rows get -1 and 0."""
import pytest
import torch

import efficient_linear_assignment_b200 as ela
from efficient_linear_assignment_b200 import _lib

pytestmark = pytest.mark.gpu


def _case(shape, dtype, seed, ties, with_prices, with_assign):
    g = torch.Generator().manual_seed(seed)
    B, N, M = shape
    if ties:  # integer costs: many tied maxima
        cost = torch.randint(0, 8, shape, generator=g).to(dtype)
    else:
        cost = torch.rand(shape, generator=g, dtype=torch.float64).to(dtype)
    pdt = torch.float64 if dtype == torch.float64 else torch.float32
    prices = None
    if with_prices:  # a few price levels, so ties survive the subtraction
        prices = (torch.randint(0, 4, (B, M), generator=g).to(pdt) * 0.25) if ties else torch.rand((B, M), generator=g).to(pdt)
    assign = None
    if with_assign:
        assign = torch.randint(0, M, (B, N), generator=g)
        assign[torch.rand((B, N), generator=g) < 0.5] = -1
    return cost, prices, assign


CASES = [
    ((4, 256, 512), torch.float32, False, False, False),
    ((2, 300, 1024), torch.float32, False, True, True),
    ((2, 300, 1024), torch.bfloat16, True, True, True),      # tie-heavy, M >= 128
    ((3, 200, 136), torch.float16, True, True, False),
    ((2, 64, 96), torch.float32, True, True, True),          # M < 128: torch.topk's introselect on ties
    ((2, 50, 40), torch.float16, True, False, True),
    ((2, 33, 10), torch.float32, True, True, False),         # rows not 16-byte aligned: scalar loads
    ((2, 64, 136), torch.float64, False, True, True),
    ((2, 64, 136), torch.float64, True, True, False),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_bids_equal_oracle(case, oracle_mod):
    shape, dtype, ties, wp, wa = CASES[case]
    cost, prices, assign = _case(shape, dtype, 100 + case, ties, wp, wa)
    eps = 1e-2
    ref_idx, ref_inc = oracle_mod.bids(cost, eps, prices, assign)
    idx, inc = ela.compute_bids(cost.cuda(), eps, None if prices is None else prices.cuda(),
                                None if assign is None else assign.cuda())
    assert torch.equal(idx.cpu(), ref_idx)
    assert torch.equal(inc.cpu(), ref_inc)


def test_bids_strided_rows_equal_oracle(oracle_mod):
    g = torch.Generator().manual_seed(7)
    wide = torch.randint(0, 5, (3, 128, 272), generator=g).float()
    cost = wide[:, :, :256]  # row stride 272 > M
    ref_idx, ref_inc = oracle_mod.bids(cost.contiguous(), 0.5)
    idx, inc = ela.compute_bids(wide.cuda()[:, :, :256], 0.5)
    assert torch.equal(idx.cpu(), ref_idx)
    assert torch.equal(inc.cpu(), ref_inc)


def test_bids_full_size_cfg2_and_cfg5_problem(oracle_mod):
    # the first round of cfg2 (every row bids against zero prices) and one
    # 8192^2 bf16 problem of cfg5 (tie-heavy integer costs)
    for cost, eps in ((ela.workloads.cfg2(), 1.0), (ela.workloads.cfg5(8, 8192)[2:3].contiguous(), 1.0 / 8193)):
        ref_idx, ref_inc = oracle_mod.bids(cost, eps)
        idx, inc = ela.compute_bids(cost.cuda(), eps)
        assert torch.equal(idx.cpu(), ref_idx)
        assert torch.equal(inc.cpu(), ref_inc)


def test_bids_unbatched_and_empty():
    c = torch.rand(16, 128).cuda()
    idx, inc = ela.compute_bids(c, 0.1)
    assert idx.shape == (16,) and inc.shape == (16,)
    idx, inc = ela.compute_bids(torch.rand(2, 0, 128).cuda(), 0.1)
    assert idx.shape == (2, 0)


def test_bids_rejects_bad_arguments():
    with pytest.raises(_lib.AuctionError):
        ela.compute_bids(torch.rand(2, 8, 1).cuda(), 0.1)   # M < 2: no second value
    with pytest.raises(_lib.AuctionError):
        ela.compute_bids(torch.rand(2, 8, 16).cuda(), float("inf"))


def test_bids_report_unsupported_when_prices_do_not_fit():
    # the problem's prices are staged in shared memory: a row longer than that
    # holds is refused with ELA_ERR_UNSUPPORTED, not run
    with pytest.raises(_lib.AuctionError) as e:
        ela.compute_bids(torch.rand(1, 8, 64000).cuda(), 0.1)
    assert e.value.status == _lib.ELA_ERR_UNSUPPORTED
