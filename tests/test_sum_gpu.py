"""GPU tests of the fused IMLE target solve (ela_auction_solve_sum): the kernel
reads C and G and forms C + lambda*G in its loads, rounded as torch evaluates
the sum in the input dtype, so it must equal the CPU oracle run on the
materialised ``C + lam * G`` bit for bit, and the IMLE backward built on it must
equal the one that solves the materialised target."""
import pytest
import torch

import efficient_linear_assignment_b200 as ela
from efficient_linear_assignment_b200 import _lib

pytestmark = pytest.mark.gpu


def _pair(shape, dtype, seed, ties=False):
    g = torch.Generator().manual_seed(seed)
    C = torch.randint(0, 6, shape, generator=g).float() if ties else torch.rand(shape, generator=g)
    G = torch.randn(shape, generator=g) * 0.3
    return C.to(dtype), G.to(dtype)


CASES = [((4, 256, 256), False), ((3, 136, 136), True), ((2, 512, 520), False), ((2, 64, 96), True),
         ((1, 1024, 1024), False)]


@pytest.mark.parametrize("path", [ela.PATH_AUTO, ela.PATH_CTA, ela.PATH_GRID])
@pytest.mark.parametrize("lam", [1.0, 0.5, 3.0])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_sum_solve_equals_oracle_on_materialised_target(case, lam, path, oracle_mod):
    shape, ties = CASES[case]
    C, G = _pair(shape, torch.float32, seed=case * 7 + int(lam * 10), ties=ties)
    target = C + lam * G  # what the reference's backward builds (torch, CPU, fp32)
    ao, po, so = oracle_mod.solve(target, 1e-2, 2000, nthreads=4)
    try:
        a, p, st, status = ela.auction_solve_sum(C.cuda(), G.cuda(), lam, [1e-2], 2000, path)
    except ela.AuctionError as e:
        if e.status == _lib.ELA_ERR_UNSUPPORTED:
            pytest.skip("size not supported on this path")
        raise
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(a.cpu(), ao) and torch.equal(p.cpu(), po)
    assert torch.equal(st[:, :2].cpu(), so[:, :2])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float64])
def test_sum_solve_rounds_like_torch_in_the_dtype(dtype, oracle_mod):
    for shape, ties in ((2, 256, 256), False), ((2, 72, 80), True):
        C, G = _pair(shape, dtype, seed=11, ties=ties)
        for lam in (1.0, 0.37):
            target = C + lam * G  # rounded twice in the dtype, as the kernel must
            ao, po, _ = oracle_mod.solve(target, 1e-2, 2000)
            a, p, _, status = ela.auction_solve_sum(C.cuda(), G.cuda(), lam, [1e-2], 2000)
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            assert torch.equal(a.cpu(), ao) and torch.equal(p.cpu(), po)


def test_cluster_path_is_refused():
    C, G = _pair((1, 256, 256), torch.float32, seed=1)
    with pytest.raises(ela.AuctionError) as ei:
        ela.auction_solve_sum(C.cuda(), G.cuda(), 1.0, [1e-2], 100, ela.PATH_CLUSTER)
    assert ei.value.status == _lib.ELA_ERR_UNSUPPORTED


@pytest.mark.parametrize("shape", [(2, 64, 64), (3, 512, 512)])
def test_imle_backward_fused_equals_materialised_target(shape, oracle_mod):
    C, G = _pair(shape, torch.float32, seed=5)
    c = C.cuda().requires_grad_(True)
    P = ela.linear_assignment(c, epsilon=1e-2, return_indices=False)
    P.backward(G.cuda())
    af, _, _ = oracle_mod.solve(C, 1e-2, 1000, nthreads=4)
    at, _, _ = oracle_mod.solve(C + G, 1e-2, 1000, nthreads=4)
    M = shape[2]
    eye = torch.eye(M)
    expect = eye[at.clamp(min=0)] * (at >= 0)[..., None] - eye[af.clamp(min=0)] * (af >= 0)[..., None]
    assert torch.equal(c.grad.cpu(), expect)
