"""GPU tests of the padded solve without a padded copy (ela_auction_solve_padded):
the kernel synthesises the reference's padding blocks (utils.py:32-105: real rows
get 1e9 on the added columns, added rows 1e9 on the real columns and 0 on the
added columns when both dimensions are padded), so its results must equal the
CPU oracle run on the explicit ``pad_input`` tensor, bit for bit, for every row
and column of the padded problem."""
import pytest
import torch

import efficient_linear_assignment_b200 as ela
from efficient_linear_assignment_b200 import _lib

pytestmark = pytest.mark.gpu

SHAPES = [(1, 13, 16), (2, 16, 21), (1, 120, 121), (2, 130, 133), (1, 133, 130), (3, 7, 9), (1, 250, 8), (2, 5, 300)]


def _cost(shape, dtype, ties):
    B, N, M = shape
    g = torch.Generator().manual_seed(N * 1000 + M)
    c = torch.randint(0, 5, (B, N, M), generator=g).float() if ties else torch.rand(B, N, M, generator=g)
    return c.to(dtype)


@pytest.mark.parametrize("path", [ela.PATH_AUTO, ela.PATH_CTA, ela.PATH_GRID])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ties", [False, True])
def test_padded_solve_equals_oracle_on_pad_input(shape, ties, path, oracle_mod):
    cost = _cost(shape, torch.float32, ties)
    padded, _ = ela.pad_input(cost)
    eps = [0.5, 1e-2]
    ao, po, so = oracle_mod.solve(padded, eps, 2000, nthreads=4)
    try:
        a, p, st, status = ela.auction_solve_padded(cost.cuda(), eps, 2000, path)
    except ela.AuctionError as e:
        if e.status == _lib.ELA_ERR_UNSUPPORTED:
            pytest.skip("size not supported on this path")
        raise
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert a.shape == ao.shape and p.shape == po.shape
    assert torch.equal(a.cpu(), ao) and torch.equal(p.cpu(), po)
    assert torch.equal(st[:, :2].cpu(), so[:, :2])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float64])
def test_padded_solve_dtypes(dtype, oracle_mod):
    """fp16 holds the 1e9 padding as +inf, bf16 rounds it: the synthesised
    values must be the ones torch.full(..., 1e9, dtype) stores."""
    for shape in ((2, 13, 21), (1, 130, 133)):
        cost = _cost(shape, dtype, ties=False)
        # pad_input itself refuses fp16 (torch.full cannot store 1e9 there); the
        # padded solve takes 1e9 rounded to the dtype, +inf: build that tensor
        padded = ela.pad_input(cost.float())[0].to(dtype) if dtype == torch.float16 else ela.pad_input(cost)[0]
        ao, po, _ = oracle_mod.solve(padded, 1e-2, 2000)
        a, p, _, status = ela.auction_solve_padded(cost.cuda(), [1e-2], 2000)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(a.cpu(), ao) and torch.equal(p.cpu(), po)


def test_cluster_path_is_refused_for_padded_shapes():
    with pytest.raises(ela.AuctionError) as ei:
        ela.auction_solve_padded(torch.rand(1, 130, 133, device="cuda"), [1e-2], 100, ela.PATH_CLUSTER)
    assert ei.value.status == _lib.ELA_ERR_UNSUPPORTED


def test_auto_pad_builds_no_padded_copy(monkeypatch, oracle_mod):
    """linear_assignment(auto_pad=True) returns unpad_result(solve(pad_input(C)))
    for the cases that used to solve a padded copy, without calling pad_input."""
    import efficient_linear_assignment_b200.utils as U
    for shape in ((2, 16, 21), (1, 120, 121), (1, 133, 130)):
        cost = _cost(shape, torch.float32, ties=True)
        padded, orig = ela.pad_input(cost)
        ao, _, _ = oracle_mod.solve(padded, 1e-2, 3000)
        expect = ela.unpad_result(ao.clamp(min=0), orig)

        def no_copy(*a, **k):
            raise AssertionError("pad_input was called")
        monkeypatch.setattr(U, "pad_input", no_copy)
        got = ela.linear_assignment(cost.cuda(), epsilon=1e-2, max_iter=3000, auto_pad=True)
        monkeypatch.undo()
        assert torch.equal(got.cpu(), expect)
