"""GPU parity: the CUDA solver against golden vectors recorded from the
reference (bit-exact assignment and prices) and against the CPU oracle."""
import numpy as np
import pytest
import torch

import efficient_linear_assignment_b200 as ela
from efficient_linear_assignment_b200 import _lib
from cases import CASES
from make_golden_io import load_golden

pytestmark = pytest.mark.gpu

PATHS = {"auto": ela.PATH_AUTO, "cta": ela.PATH_CTA, "grid": ela.PATH_GRID, "cluster": ela.PATH_CLUSTER}
BIG = {"cfg2_fixed", "cfg2_escale", "cfg2_maxiter10", "cfg3_f16", "cfg3_bf16"}


def gpu_solve(cost, eps, max_iter, path):
    try:
        a, p, st = ela.solve(cost.cuda(), eps, max_iter, path=path)
    except ela.AuctionError as e:
        if e.status == _lib.ELA_ERR_UNSUPPORTED:
            pytest.skip("size not supported on this path")
        raise
    return a.cpu(), p.cpu(), st.cpu()


@pytest.mark.parametrize("path", sorted(PATHS))
@pytest.mark.parametrize("name", sorted(CASES))
def test_golden_bit_exact(name, path):
    make, eps, max_iter = CASES[name]
    if path == "cta" and name in BIG:
        pytest.skip("one-CTA path on a 4096^2 problem is correct but slow; covered by auto/grid")
    g = load_golden(name)
    a, p, st = gpu_solve(make(), eps, max_iter, PATHS[path])
    assert np.array_equal(a.numpy(), g["assign"].astype(np.int64)), \
        f"{int((a.numpy() != g['assign']).sum())} rows differ"
    assert np.array_equal(p.numpy(), g["prices"])
    assert torch.equal(st[:, 3], (a == -1).sum(1))


@pytest.mark.parametrize("path", ["cta", "grid", "cluster"])
@pytest.mark.parametrize("seed", range(4))
def test_random_vs_oracle(seed, path, oracle_mod):
    g = torch.Generator().manual_seed(1000 + seed)
    B = [1, 3, 5, 2][seed]
    N = [256, 64, 136, 512][seed]
    M = [256, 128, 136, 520][seed]
    cost = torch.rand(B, N, M, generator=g)
    if seed % 2:
        cost = (cost * 8).floor()  # integer costs: many ties
    eps = [1e-2, 1.0 / (N + 1), [0.5, 0.05, 1e-3], 1e-3][seed]
    a, p, st = gpu_solve(cost, eps, 1000, PATHS[path])
    ao, po, so = oracle_mod.solve(cost, eps, 1000, nthreads=4)
    assert torch.equal(a, ao)
    assert torch.equal(p, po)
    assert torch.equal(st[:, :2], so[:, :2])


def test_cfg4_full_batch_vs_oracle(oracle_mod):
    cost = ela.workloads.cfg4()
    a, p, st = gpu_solve(cost, 1e-2, 1000, ela.PATH_AUTO)
    ao, po, so = oracle_mod.solve(cost, 1e-2, 1000, nthreads=8)
    assert torch.equal(a, ao) and torch.equal(p, po)
    assert int(st[:, 1].sum()) == int(so[:, 1].sum())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float64])
def test_dtypes_vs_oracle(dtype, oracle_mod):
    cost = ela.workloads.uniform(2, 256, 256, seed=77, dtype=dtype)
    for path in (ela.PATH_CTA, ela.PATH_GRID, ela.PATH_CLUSTER):
        a, p, _ = gpu_solve(cost, 1e-3, 1000, path)
        ao, po, _ = oracle_mod.solve(cost, 1e-3, 1000)
        assert torch.equal(a, ao) and torch.equal(p, po)


def test_unaligned_rows_use_scalar_loads(oracle_mod):
    # stride_n = M + 1 elements: rows are not 16-byte aligned
    full = ela.workloads.uniform(2, 64, 73, seed=5)
    cost = full[:, :, :72]
    a, p, _ = ela.solve(cost.cuda(), 1e-3, 1000)
    ao, po, _ = oracle_mod.solve(cost.contiguous(), 1e-3, 1000)
    assert torch.equal(a.cpu(), ao) and torch.equal(p.cpu(), po)


@pytest.mark.parametrize("cs", [16, 8, 4, 2])
@pytest.mark.parametrize("team", ["1", "auto"])
def test_cluster_shapes_vs_oracle(cs, team, monkeypatch, oracle_mod):
    """Every cluster size, with one cluster per problem (bids over distributed
    shared memory) and with teams of clusters (bids over global memory)."""
    monkeypatch.setenv("ELA_CLUSTER_SIZE", str(cs))
    if team == "1":
        monkeypatch.setenv("ELA_CLUSTERS_PER_PROBLEM", "1")
    cases = [
        (ela.workloads.uniform(1, 1024, 1024, seed=21), 1e-3),            # large then small rounds
        (ela.workloads.uniform(3, 256, 264, seed=22, dtype=torch.bfloat16), 1e-2),
        (ela.workloads.cfg5(2, 512), [16.0, 1.0, 1.0 / 513]),            # tie-heavy, epsilon schedule
    ]
    for cost, eps in cases:
        a, p, st = gpu_solve(cost, eps, 1000, ela.PATH_CLUSTER)
        ao, po, so = oracle_mod.solve(cost, eps, 1000, nthreads=4)
        assert torch.equal(a, ao) and torch.equal(p, po)
        assert torch.equal(st[:, :2], so[:, :2])


def test_cfg5_full_size_problem_vs_oracle(oracle_mod):
    """One 8192 x 8192 bf16 problem of config 5 (integer costs, zero rows,
    constant columns: ties everywhere; 1000 rounds of price war), bit-exact."""
    import os
    cost = ela.workloads.cfg5(8, 8192)[3:4].contiguous()
    a, p, st = gpu_solve(cost, 1.0 / 8193, 1000, ela.PATH_AUTO)
    ao, po, so = oracle_mod.solve(cost, 1.0 / 8193, 1000, nthreads=os.cpu_count() or 4)
    assert torch.equal(a, ao) and torch.equal(p, po)
    assert torch.equal(st[:, :2], so[:, :2])
    assert int(st[0, 3]) == int((a == -1).sum())


def test_custom_op_traces_under_torch_compile():
    cost = ela.workloads.uniform(2, 128, 128, seed=9).cuda()

    def f(c):
        a, p, st, status = ela.auction_solve_op(c, [1e-2], 1000, 0)
        return a, p

    a0, p0 = f(cost)
    a1, p1 = torch.compile(f, backend="aot_eager", fullgraph=True)(cost)
    assert torch.equal(a0, a1) and torch.equal(p0, p1)
