"""GPU tests of the public API, ported from the reference's auction tests
(tests/test_all.py, tests/test_robustness.py) plus the IMLE backward."""
import pytest
import scipy.optimize
import torch

import efficient_linear_assignment_b200 as ela
from efficient_linear_assignment_b200 import _lib

pytestmark = pytest.mark.gpu
dev = "cuda"


def total_cost(cost, idx):
    B, N, _ = cost.shape
    return cost[torch.arange(B)[:, None], torch.arange(N)[None], idx].sum(1)


def test_simple_match_vs_scipy():  # reference tests/test_all.py:19-44
    cost = ela.workloads.uniform(2, 8, 8, seed=3).to(dev)
    idx = ela.linear_assignment(cost, epsilon=1e-3, max_iter=2000)
    for b in range(2):
        r, c = scipy.optimize.linear_sum_assignment(cost[b].cpu().numpy())
        assert total_cost(cost[b:b + 1], idx[b:b + 1]).item() <= cost[b].cpu().numpy()[r, c].sum() + 1e-1


@pytest.mark.parametrize("N", [128, 136, 144, 256])
def test_correctness_vs_hungarian(N):  # reference tests/test_robustness.py:10-60
    cost = ela.workloads.uniform(2, N, N, seed=N).to(dev)
    idx = ela.linear_assignment(cost, epsilon=1e-3, max_iter=5000)
    mine = total_cost(cost, idx).cpu()
    for b in range(2):
        r, c = scipy.optimize.linear_sum_assignment(cost[b].double().cpu().numpy())
        opt = cost[b].cpu().numpy()[r, c].sum()
        assert mine[b].item() - opt <= 1.5 * N * 1e-3
        assert len(torch.unique(idx[b])) == N


def test_degenerate_cases():  # reference tests/test_robustness.py:63-99
    for cost in (torch.zeros(2, 32, 32, device=dev), torch.full((2, 32, 32), 10.0, device=dev)):
        idx = ela.linear_assignment(cost, max_iter=1000)
        for b in range(2):
            assert len(torch.unique(idx[b])) == 32


def test_batched_correctness():  # reference tests/test_robustness.py:101-126
    cost = torch.rand(4, 32, 32, device=dev)
    cost[0] = 100.0
    cost[0].diagonal().zero_()
    idx = ela.linear_assignment(cost, max_iter=2000)
    assert torch.equal(idx[0], torch.arange(32, device=dev))
    for b in range(1, 4):
        assert len(torch.unique(idx[b])) == 32


def test_unbatched_input_and_one_hot():
    cost = ela.workloads.uniform(1, 64, 64, seed=9)[0].to(dev)
    idx = ela.linear_assignment(cost, epsilon=1e-3)
    P = ela.linear_assignment(cost, epsilon=1e-3, return_indices=False)
    assert idx.shape == (64,) and P.shape == (64, 64)
    assert torch.equal(P.argmax(1), idx)
    assert P.dtype == cost.dtype


def test_imle_gradient_flows():  # reference tests/test_all.py:46-114
    cost = torch.randn(1, 8, 8, device=dev, dtype=torch.double, requires_grad=True)
    out = ela.linear_assignment(cost, epsilon=1e-3, max_iter=200, return_indices=False)
    (out * cost).sum().backward()
    assert cost.grad is not None and (cost.grad != 0).any()


def test_imle_backward_is_target_minus_forward(oracle_mod):
    g = torch.Generator().manual_seed(4)
    C = torch.rand(2, 16, 16, generator=g)
    G = torch.randn(2, 16, 16, generator=g)
    c = C.to(dev).requires_grad_(True)
    P = ela.linear_assignment(c, epsilon=1e-3, return_indices=False)
    P.backward(G.to(dev))
    af, _, _ = oracle_mod.solve(C, 1e-3, 1000)
    at, _, _ = oracle_mod.solve(C + G, 1e-3, 1000)
    eye = torch.eye(16)
    expect = eye[at.clamp(min=0)] * (at >= 0)[..., None] - eye[af.clamp(min=0)] * (af >= 0)[..., None]
    assert torch.equal(c.grad.cpu(), expect)


def test_unassigned_rows_map_to_zero():
    cost = ela.workloads.uniform(1, 16, 8, seed=13).to(dev)
    a, _, st = ela.solve(cost, 1e-2, 50)
    idx = ela.linear_assignment(cost, epsilon=1e-2, max_iter=50)
    assert (a == -1).any()
    assert torch.equal(idx, a.clamp(min=0))


def test_max_iter_zero():
    cost = torch.rand(2, 16, 16, device=dev)
    for path in (ela.PATH_CTA, ela.PATH_GRID):
        a, p, st = ela.solve(cost, 1e-2, 0, path=path)
        assert (a == -1).all() and (p == 0).all() and (st[:, 3] == 16).all()


def test_nondefault_stream():
    cost = ela.workloads.uniform(3, 128, 128, seed=2).to(dev)
    ref, _, _ = ela.solve(cost, 1e-2)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a, _, _ = ela.solve(cost, 1e-2)
    s.synchronize()
    assert torch.equal(a, ref)


def test_wait_timeout_reports_status_and_context_survives():
    """A barrier whose arrival never comes ends in ELA_ERR_TIMEOUT, not a hang."""
    lib = _lib.load()
    cost = ela.workloads.uniform(1, 512, 512, seed=3).to(dev)
    lib.ela_auction_set_wait_limit_ns(20_000_000)  # 20 ms
    lib.ela_auction_debug_skip_arrive(1)
    try:
        with pytest.raises(ela.AuctionError) as ei:
            ela.solve(cost, 1e-2, path=ela.PATH_GRID)
        assert ei.value.status == _lib.ELA_ERR_TIMEOUT
    finally:
        lib.ela_auction_debug_skip_arrive(0)
        lib.ela_auction_set_wait_limit_ns(2_000_000_000)
    a, _, _ = ela.solve(cost, 1e-2, path=ela.PATH_GRID)
    b, _, _ = ela.solve(cost, 1e-2, path=ela.PATH_CTA)
    assert torch.equal(a, b)


def test_multi_device_sharding_matches_single_solve():
    from efficient_linear_assignment_b200.sharding import solve_multi_device
    cost = ela.workloads.cfg4(B=12, N=128).to(dev)
    ref_a, ref_p, _ = ela.solve(cost, 1e-2)
    devs = [torch.device("cuda", i) for i in range(torch.cuda.device_count())]
    a, p = solve_multi_device(cost, devs, epsilon=1e-2)  # default: no synchronisation between devices
    assert torch.equal(a, ref_a) and torch.equal(p, ref_p)
    a2, p2 = solve_multi_device(cost, devs, lambda c: ela.solve(c, 1e-2, return_status=True, check=False))
    assert torch.equal(a2, ref_a) and torch.equal(p2, ref_p)


@pytest.mark.parametrize("shape", [(2, 13, 21), (1, 16, 21), (1, 13, 16), (3, 7, 9)])
def test_auto_pad_equals_explicit_padding(shape):
    """auto_pad returns the real rows of the solve of pad_input(cost)."""
    B, N, M = shape
    g = torch.Generator().manual_seed(N * 100 + M)
    cost = torch.rand(B, N, M, generator=g).to(dev)
    padded, orig = ela.pad_input(cost)
    expect = ela.unpad_result(ela.linear_assignment(padded, epsilon=1e-3, max_iter=2000), orig)
    got = ela.linear_assignment(cost, epsilon=1e-3, max_iter=2000, auto_pad=True)
    assert torch.equal(got, expect)
    with pytest.raises(ValueError):
        ela.linear_assignment(cost, epsilon=1e-3)


def test_cluster_team_wait_timeout_reports_status(monkeypatch):
    """The global-memory exchange between the clusters of a team is bounded too."""
    lib = _lib.load()
    monkeypatch.setenv("ELA_CLUSTER_SIZE", "4")  # a team of several clusters for one problem
    cost = ela.workloads.uniform(1, 2048, 2048, seed=6).to(dev)
    lib.ela_auction_set_wait_limit_ns(20_000_000)
    lib.ela_auction_debug_skip_arrive(1)
    try:
        with pytest.raises(ela.AuctionError) as ei:
            ela.solve(cost, 1e-2, path=ela.PATH_CLUSTER)
        assert ei.value.status == _lib.ELA_ERR_TIMEOUT
    finally:
        lib.ela_auction_debug_skip_arrive(0)
        lib.ela_auction_set_wait_limit_ns(2_000_000_000)
    a, _, _ = ela.solve(cost, 1e-2, path=ela.PATH_CLUSTER)
    b, _, _ = ela.solve(cost, 1e-2, path=ela.PATH_GRID)
    assert torch.equal(a, b)


@pytest.mark.parametrize("shape,path", [((3, 64, 64), ela.PATH_AUTO), ((1, 1024, 1024), ela.PATH_CLUSTER),
                                        ((4, 256, 264), ela.PATH_GRID)])
def test_eager_entry_equals_custom_op(shape, path):
    """auction_solve (the eager call behind linear_assignment) and the registered
    ela::auction_solve op are one computation: identical outputs, repeated calls
    (cached launch plan) included."""
    cost = ela.workloads.uniform(*shape, seed=sum(shape)).to(dev)
    eps = [0.1, 1e-2]
    ref = ela.auction_solve_op(cost, eps, 1000, path)
    for _ in range(2):
        got = ela.auction_solve(cost, eps, 1000, path)
        torch.cuda.synchronize()
        assert int(got[3].item()) == 0
        for g, r in zip(got, ref):
            assert torch.equal(g, r)


def test_host_tensor_is_solved_on_the_gpu(oracle_mod):
    # the reference's linear_assignment takes CPU tensors; here a host cost is
    # copied to the current GPU, solved by the same kernels, and the indices
    # come back on the host, equal to the oracle's
    cost = ela.workloads.cfg1()
    idx = ela.linear_assignment(cost, epsilon=1e-2)
    assert idx.device.type == "cpu"
    a, _, _ = oracle_mod.solve(cost, 1e-2, 1000)
    assert torch.equal(idx, a.clamp(min=0))
    a2, p2 = ela.AuctionB200(1e-2, 1000).solve(cost)
    assert a2.device.type == "cpu" and p2.device.type == "cpu" and torch.equal(a2, a)
    # auto_pad through the host path
    odd = torch.rand(2, 20, 21, generator=torch.Generator().manual_seed(3))
    assert torch.equal(ela.linear_assignment(odd, auto_pad=True),
                       ela.linear_assignment(odd.cuda(), auto_pad=True).cpu())


def test_host_tensor_one_hot_and_backward_match_device():
    g = torch.Generator().manual_seed(12)
    base = torch.rand(2, 64, 64, generator=g)
    grad = torch.randn(2, 64, 64, generator=g)
    c_host = base.clone().requires_grad_(True)
    P_host = ela.linear_assignment(c_host, epsilon=1e-2, return_indices=False)
    (P_host * grad).sum().backward()
    c_dev = base.cuda().requires_grad_(True)
    P_dev = ela.linear_assignment(c_dev, epsilon=1e-2, return_indices=False)
    (P_dev * grad.cuda()).sum().backward()
    assert P_host.device.type == "cpu" and torch.equal(P_host, P_dev.cpu())
    assert torch.equal(c_host.grad, c_dev.grad.cpu())
