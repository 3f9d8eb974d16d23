"""GPU test of ela_auction_solve_noalloc, the entry point for callers that
cannot allocate device memory (a host that pre-reserves all GPU memory in its
own pool, code that must avoid cudaMalloc's implicit synchronisation, or a
foreign-language binding without a device allocator).  It must give exactly
the results of ela_auction_solve, call after call, while its scratch comes
from the library's fixed device array.

Kept in its own file, collected last, so that a run stopping at the first
failure has already run every other test.
"""
import ctypes

import pytest
import torch

import efficient_linear_assignment_b200 as ela
from efficient_linear_assignment_b200 import _lib
from efficient_linear_assignment_b200.solver import DTYPE_CODE

pytestmark = pytest.mark.gpu


def _outputs(B, N, M, dtype, dev):
    pdt = torch.float64 if dtype == torch.float64 else torch.float32
    return (torch.full((B, N), -7, dtype=torch.int64, device=dev), torch.full((B, M), -1.0, dtype=pdt, device=dev),
            torch.full((B, 4), -1, dtype=torch.int64, device=dev), torch.full((1,), -1, dtype=torch.int32, device=dev))


def _call(fn_name, cost, eps, max_iter, path, ws=None, tie_rule=0):
    lib = _lib.load()
    B, N, M = cost.shape
    a, p, st, status = _outputs(B, N, M, cost.dtype, cost.device)
    e = (ctypes.c_double * len(eps))(*eps)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = [ctypes.c_void_p(cost.data_ptr()), DTYPE_CODE[cost.dtype], B, N, M, cost.stride(0), cost.stride(1),
              e, len(eps), max_iter, path, tie_rule, ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(p.data_ptr()),
              ctypes.c_void_p(st.data_ptr()), ctypes.c_void_p(status.data_ptr())]
    if fn_name == "ela_auction_solve":
        rc = lib.ela_auction_solve(*common, ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream)
    else:
        rc = lib.ela_auction_solve_noalloc(*common, stream)
    torch.cuda.synchronize()
    return rc, a, p, st, status


@pytest.mark.parametrize("shape,dtype,eps,path,tie_rule,team", [
    ((1, 512, 512), torch.float32, [1e-2], ela.PATH_GRID, 0, None),
    ((3, 1024, 1024), torch.float32, [1.0, 0.25, 0.0625, 1e-2], ela.PATH_GRID, 0, None),
    ((2, 256, 264), torch.bfloat16, [1e-3], ela.PATH_GRID, 1, None),
    ((4, 128, 128), torch.float32, [1e-2], ela.PATH_CTA, 0, None),
    # the cluster path that AUTO picks for large problems: one problem shared
    # by a team of clusters (exchange segments in the scratch), then one
    # cluster per problem
    ((1, 2048, 2048), torch.float32, [1.0, 0.1, 1e-2], ela.PATH_CLUSTER, 0, None),
    ((2, 1024, 1024), torch.bfloat16, [1e-2], ela.PATH_CLUSTER, 0, "1"),
])
def test_noalloc_matches_workspace_entry_point_twice(shape, dtype, eps, path, tie_rule, team, monkeypatch):
    if team is not None:
        monkeypatch.setenv("ELA_CLUSTERS_PER_PROBLEM", team)
    B, N, M = shape
    cost = ela.workloads.uniform(B, N, M, seed=N + B, dtype=dtype).cuda()
    lib = _lib.load()
    ws_bytes = lib.ela_auction_workspace_bytes(DTYPE_CODE[dtype], B, N, M, path)
    assert 0 < ws_bytes <= (4 << 20)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    rc, a0, p0, s0, st0 = _call("ela_auction_solve", cost, eps, 1000, path, ws, tie_rule)
    assert rc == 0 and st0.item() == 0
    for _ in range(2):  # the shared array keeps the last call's contents
        rc, a, p, s, st = _call("ela_auction_solve_noalloc", cost, eps, 1000, path, tie_rule=tie_rule)
        assert rc == 0 and st.item() == 0
        assert torch.equal(a, a0) and torch.equal(p, p0) and torch.equal(s, s0)


def test_noalloc_rejects_scratch_beyond_its_limit():
    B, N, M = 8, 16384, 16  # exchange segments need more than 4 MiB
    lib = _lib.load()
    need = lib.ela_auction_workspace_bytes(0, B, N, M, ela.PATH_GRID)
    assert need > (4 << 20)
    cost = torch.rand(B, N, M, device="cuda")
    rc, a, _, _, _ = _call("ela_auction_solve_noalloc", cost, [1e-2], 10, ela.PATH_GRID)
    assert rc == _lib.ELA_ERR_UNSUPPORTED
    assert (a == -7).all()  # nothing was run
