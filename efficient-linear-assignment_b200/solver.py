"""Solver backend over the CUDA library.

``AuctionB200`` is the drop-in for the reference's backend plug-in
(``AuctionTorch`` / ``AuctionCPPCCUDA``: ``cls(epsilon, max_iter).solve(cost)
-> (assignment (B,N) int64 with -1 = unassigned, prices (B,M))``,
src/efficient_linear_assignment/auction/api.py:7-47,56-61 and
src/efficient_linear_assignment/auction/cpp_backend.py:18-40).  The solve is
the C++ torch operator ``torch.ops.ela_native.auction_solve``
(csrc/ela_torch_op.cpp), which calls ``ela_auction_solve`` through the C ABI
on the current stream.  The other entry points (padded, fused sum, implicit)
call the C ABI through ctypes.
"""
from __future__ import annotations

import ctypes
import os
from typing import Sequence, Tuple, Union

import torch

from . import _lib

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}

EpsArg = Union[float, Sequence[float]]


def _as_schedule(epsilon: EpsArg) -> list[float]:
    if isinstance(epsilon, (int, float)):
        return [float(epsilon)]
    sched = [float(e) for e in epsilon]
    if not sched:
        raise ValueError("epsilon schedule is empty")
    return sched


_op_loaded = False


def _native_op():
    """torch.ops.ela_native.auction_solve, the C++ operator over the C ABI
    (csrc/ela_torch_op.cpp, built in-tree next to libela_auction.so)."""
    global _op_loaded
    if not _op_loaded:
        path = os.path.join(os.path.dirname(_lib.LIB_PATH), "libela_torch_op.so")
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing: build it with __graft_entry__.build() (no CPU fallback exists)")
        _lib.load()
        torch.ops.load_library(path)
        _op_loaded = True
    return torch.ops.ela_native.auction_solve


def auction_solve(cost: torch.Tensor, eps: list[float], max_iter: int, path: int, tie_rule: int = 0) -> Tuple[
        torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(B,N,M) CUDA cost -> (assignment int64 (B,N), prices (B,M), stats int64 (B,4), status int32 (1,)).

    One call of the C++ operator ``torch.ops.ela_native.auction_solve``
    (device guard, checks, outputs from the caching allocator, one
    ``ela_auction_solve`` on the current stream; ~20 us of host time), no
    synchronisation: the device status word is read by the caller.  A return
    code other than ELA_OK from the library raises AuctionError.
    tie_rule: ``_lib.TIE_HIGHEST_ROW`` (0, the reference's election) or
    ``_lib.TIE_LOWEST_ROW`` (1).
    """
    if cost.device.type != "cuda":
        raise RuntimeError("ela::auction_solve needs a CUDA tensor (there is no CPU path)")
    if cost.dtype not in DTYPE_CODE:
        raise TypeError(f"unsupported cost dtype {cost.dtype}")
    if cost.dim() != 3:
        raise ValueError("cost must be (B, N, M)")
    assign, prices, stats, status, rc = _native_op()(cost, [float(e) for e in eps], int(max_iter), int(path),
                                                     int(tie_rule))
    _lib.check(int(rc), "ela_auction_solve")
    return assign, prices, stats, status


def auction_solve_padded(cost: torch.Tensor, eps: list[float], max_iter: int, path: int = 0, tie_rule: int = 0,
                         multiple: int = 8) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Solve ``pad_input(cost, multiple)`` without building it (C ABI
    ``ela_auction_solve_padded``): the kernel synthesises the reference's
    padding blocks (utils.py:32-105) in its loaders.  Returns the padded
    problem's (assignment (B,N'), prices (B,M'), stats, status) like
    ``auction_solve``; ``assignment[:, :N]`` is what ``unpad_result`` keeps.
    No synchronisation.
    """
    if cost.device.type != "cuda":
        raise RuntimeError("ela_auction_solve_padded needs a CUDA tensor (there is no CPU path)")
    code = DTYPE_CODE.get(cost.dtype)
    if code is None:
        raise TypeError(f"unsupported cost dtype {cost.dtype}")
    if cost.dim() != 3:
        raise ValueError("cost must be (B, N, M)")
    if cost.stride(2) != 1:
        cost = cost.contiguous()
    if dev_index(cost) != torch.cuda.current_device():
        with torch.cuda.device(cost.device):
            return auction_solve_padded(cost, eps, max_iter, path, tie_rule, multiple)
    lib = _lib.load()
    B, N, M = cost.shape
    Np, Mp = -(-N // multiple) * multiple, -(-M // multiple) * multiple
    dev = cost.device
    pdt = torch.float64 if code == 3 else torch.float32
    assign = torch.empty((B, Np), dtype=torch.int64, device=dev)
    prices = torch.empty((B, Mp), dtype=pdt, device=dev)
    stats = torch.empty((B, 4), dtype=torch.int64, device=dev)
    status = torch.empty((1,), dtype=torch.int32, device=dev)
    ws_bytes = lib.ela_auction_workspace_bytes(code, B, Np, Mp, int(path))
    if ws_bytes == 0:
        _lib.check(_lib.ELA_ERR_UNSUPPORTED, f"ela_auction_workspace_bytes(B={B}, N={Np}, M={Mp}, path={path})")
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
    e = (ctypes.c_double * len(eps))(*eps)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.ela_auction_solve_padded(
        cost.data_ptr(), code, B, N, M, cost.stride(0), cost.stride(1), int(multiple), e, len(eps), int(max_iter),
        int(path), int(tie_rule), assign.data_ptr(), prices.data_ptr(), stats.data_ptr(), status.data_ptr(),
        ws.data_ptr(), ws_bytes, stream)
    _lib.check(rc, "ela_auction_solve_padded")
    return assign, prices, stats, status


def auction_solve_sum(cost: torch.Tensor, grad: torch.Tensor, lam: float, eps: list[float], max_iter: int,
                      path: int = 0, tie_rule: int = 0) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Solve ``cost + lam * grad`` without materialising it (C ABI
    ``ela_auction_solve_sum``): the kernel reads both tensors and rounds the sum
    as torch does in their dtype.  Same outputs as ``auction_solve`` on the
    materialised sum.  Raises AuctionError(ELA_ERR_UNSUPPORTED) for sizes that
    only the cluster kernel runs.  No synchronisation.
    """
    if cost.device.type != "cuda" or grad.device != cost.device:
        raise RuntimeError("ela_auction_solve_sum needs cost and grad on one CUDA device")
    if grad.shape != cost.shape or grad.dtype != cost.dtype:
        raise ValueError("grad must have cost's shape and dtype")
    code = DTYPE_CODE.get(cost.dtype)
    if code is None:
        raise TypeError(f"unsupported cost dtype {cost.dtype}")
    cost, grad = cost.contiguous(), grad.contiguous()
    if dev_index(cost) != torch.cuda.current_device():
        with torch.cuda.device(cost.device):
            return auction_solve_sum(cost, grad, lam, eps, max_iter, path, tie_rule)
    lib = _lib.load()
    B, N, M = cost.shape
    dev = cost.device
    pdt = torch.float64 if code == 3 else torch.float32
    assign = torch.empty((B, N), dtype=torch.int64, device=dev)
    prices = torch.empty((B, M), dtype=pdt, device=dev)
    stats = torch.empty((B, 4), dtype=torch.int64, device=dev)
    status = torch.empty((1,), dtype=torch.int32, device=dev)
    if B == 0 or N == 0:
        prices.zero_(); stats.zero_(); status.zero_()
        return assign, prices, stats, status
    ws_bytes = lib.ela_auction_workspace_bytes(code, B, N, M, int(path))
    if ws_bytes == 0:
        _lib.check(_lib.ELA_ERR_UNSUPPORTED, f"ela_auction_workspace_bytes(B={B}, N={N}, M={M}, path={path})")
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
    e = (ctypes.c_double * len(eps))(*eps)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.ela_auction_solve_sum(
        cost.data_ptr(), grad.data_ptr(), float(lam), code, B, N, M, cost.stride(0), cost.stride(1), e, len(eps),
        int(max_iter), int(path), int(tie_rule), assign.data_ptr(), prices.data_ptr(), stats.data_ptr(),
        status.data_ptr(), ws.data_ptr(), ws_bytes, stream)
    _lib.check(rc, "ela_auction_solve_sum")
    return assign, prices, stats, status


def _implicit_args(Q: torch.Tensor, K: torch.Tensor):
    if Q.device.type != "cuda" or K.device != Q.device:
        raise RuntimeError("solve_implicit needs Q and K on one CUDA device")
    if Q.dtype != K.dtype or Q.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("Q and K must both be bfloat16 or both float16")
    squeeze = Q.dim() == 2
    if squeeze:
        Q, K = Q.unsqueeze(0), K.unsqueeze(0)
    if Q.dim() != 3 or K.dim() != 3 or Q.shape[0] != K.shape[0] or Q.shape[2] != K.shape[2]:
        raise ValueError("Q must be (B, N, D) and K (B, M, D)")
    return Q.contiguous(), K.contiguous(), squeeze


def solve_implicit(Q: torch.Tensor, K: torch.Tensor, epsilon: EpsArg = 1e-2, max_iter: int = 1000,
                   tie_rule: int = _lib.TIE_HIGHEST_ROW, check: bool = True):
    """Auction on the implicit cost C = Q K^T (minimised), cost tiles computed
    on the tensor cores every round and never stored (C ABI
    ``ela_auction_solve_implicit``).  Q (B,N,D), K (B,M,D) (or unbatched),
    bf16 or fp16, D a multiple of 16 up to 256, 128 <= M <= 512.  Returns
    (assignment (B,N) int64 with -1 unassigned, prices (B,M) fp32, stats)."""
    Q, K, squeeze = _implicit_args(Q, K)
    sched = _as_schedule(epsilon)
    B, N, D = Q.shape
    M = K.shape[1]
    dev = Q.device
    with torch.cuda.device(dev):
        lib = _lib.load()
        assign = torch.empty((B, N), dtype=torch.int64, device=dev)
        prices = torch.empty((B, M), dtype=torch.float32, device=dev)
        stats = torch.zeros((B, 4), dtype=torch.int64, device=dev)
        status = torch.empty((1,), dtype=torch.int32, device=dev)
        e = (ctypes.c_double * len(sched))(*sched)
        rc = lib.ela_auction_solve_implicit(Q.data_ptr(), K.data_ptr(), DTYPE_CODE[Q.dtype], B, N, M, D, e, len(sched),
                                            int(max_iter), int(tie_rule), assign.data_ptr(), prices.data_ptr(),
                                            stats.data_ptr(), status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(rc, "ela_auction_solve_implicit")
        if check:
            _lib.check(int(status.item()), "implicit auction kernel")
    if squeeze:
        return assign[0], prices[0], stats[0]
    return assign, prices, stats


def compute_bids(cost: torch.Tensor, epsilon: float, prices: torch.Tensor | None = None,
                 assignment: torch.Tensor | None = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """One round's bids: the reference's ``compute_bids`` (src/csrc/interface.cpp:31-40)
    through the C ABI ``ela_auction_compute_bids``.  cost (B,N,M) or (N,M) CUDA
    tensor (fp32/fp16/bf16/fp64, any row stride); prices (B,M) (fp32, fp64 for
    fp64 costs; None = zeros); assignment (B,N) int64 (None = every row bids).
    Returns (best_idx int64 (B,N), increments (B,N)): the column torch.topk
    picks on -cost - prices and (v1 - v2) + epsilon for rows whose assignment
    is -1; -1 and 0 for the others."""
    squeeze = cost.dim() == 2
    if squeeze:
        cost = cost.unsqueeze(0)
    if cost.dim() != 3 or not cost.is_cuda or cost.dtype not in DTYPE_CODE:
        raise ValueError("compute_bids: cost must be a (B,N,M) CUDA tensor of fp32/fp16/bf16/fp64")
    if cost.stride(2) != 1:
        cost = cost.contiguous()
    B, N, M = cost.shape
    dev = cost.device
    pdt = torch.float64 if cost.dtype == torch.float64 else torch.float32
    if prices is not None:
        prices = prices.reshape(B, M).to(device=dev, dtype=pdt).contiguous()
    if assignment is not None:
        assignment = assignment.reshape(B, N).to(device=dev, dtype=torch.int64).contiguous()
    with torch.cuda.device(dev):
        lib = _lib.load()
        idx = torch.empty((B, N), dtype=torch.int64, device=dev)
        inc = torch.empty((B, N), dtype=pdt, device=dev)
        rc = lib.ela_auction_compute_bids(cost.data_ptr(), DTYPE_CODE[cost.dtype], B, N, M, cost.stride(0),
                                          cost.stride(1), None if prices is None else prices.data_ptr(),
                                          None if assignment is None else assignment.data_ptr(), float(epsilon),
                                          idx.data_ptr(), inc.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(rc, "ela_auction_compute_bids")
    if squeeze:
        return idx[0], inc[0]
    return idx, inc


def implicit_costs(Q: torch.Tensor, K: torch.Tensor) -> torch.Tensor:
    """The (B,N,M) fp32 costs ``solve_implicit`` uses, written out by the same
    tensor-core instructions (C ABI ``ela_auction_implicit_costs``)."""
    Q, K, squeeze = _implicit_args(Q, K)
    B, N, D = Q.shape
    M = K.shape[1]
    dev = Q.device
    with torch.cuda.device(dev):
        lib = _lib.load()
        out = torch.empty((B, N, M), dtype=torch.float32, device=dev)
        status = torch.empty((1,), dtype=torch.int32, device=dev)
        rc = lib.ela_auction_implicit_costs(Q.data_ptr(), K.data_ptr(), DTYPE_CODE[Q.dtype], B, N, M, D, out.data_ptr(),
                                            status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(rc, "ela_auction_implicit_costs")
        _lib.check(int(status.item()), "implicit costs kernel")
    return out[0] if squeeze else out


def dev_index(t: torch.Tensor) -> int:
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def auction_solve_op(cost: torch.Tensor, eps: list[float], max_iter: int, path: int, tie_rule: int = 0) -> Tuple[
        torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """The registered operator itself (``torch.ops.ela_native.auction_solve``),
    for torch.compile graphs: (B,N,M) CUDA cost -> (assignment, prices, stats, status)."""
    assign, prices, stats, status, rc = _native_op()(cost, [float(e) for e in eps], int(max_iter), int(path),
                                                     int(tie_rule))
    if isinstance(rc, int):  # eager call; traced graphs carry rc as a symbolic int
        _lib.check(rc, "ela_auction_solve")
    return assign, prices, stats, status


def _register_fake():
    try:
        _native_op()
    except ImportError:
        return

    @torch.library.register_fake("ela_native::auction_solve")
    def _(cost, eps, max_iter, path, tie_rule):
        B, N, M = cost.shape
        pdt = torch.float64 if cost.dtype == torch.float64 else torch.float32
        return (cost.new_empty((B, N), dtype=torch.int64), cost.new_empty((B, M), dtype=pdt),
                cost.new_empty((B, 4), dtype=torch.int64), cost.new_empty((1,), dtype=torch.int32), 0)


_register_fake()


def solve(cost: torch.Tensor, epsilon: EpsArg = 1e-2, max_iter: int = 1000, path: int = _lib.PATH_AUTO,
          check: bool = True, return_status: bool = False, tie_rule: int = _lib.TIE_HIGHEST_ROW):
    """Solve a (B,N,M) or (N,M) CUDA cost tensor.

    epsilon: the reference's constant epsilon, or a schedule (one full solve per
    value, each starting from the previous prices).
    tie_rule: which row wins among the bids on a column within 1e-5 of its new
    price, ``TIE_HIGHEST_ROW`` (the reference) or ``TIE_LOWEST_ROW``.
    Returns (assignment, prices, stats), plus the int32 device status word when
    ``return_status``; with ``check`` the device status is read back (one
    synchronisation) and a device-side error raises AuctionError.
    """
    squeeze = cost.dim() == 2
    if squeeze:
        cost = cost.unsqueeze(0)
    if max_iter < 0:
        raise ValueError("max_iter must be >= 0")
    sched = _as_schedule(epsilon)
    if any(not (e > 0.0) or e == float("inf") for e in sched):
        raise ValueError("every epsilon must be finite and > 0")
    # the registered operator while torch.compile traces, else the eager
    # wrapper around the same operator
    fn = auction_solve_op if torch.compiler.is_compiling() else auction_solve
    if tie_rule not in (_lib.TIE_HIGHEST_ROW, _lib.TIE_LOWEST_ROW):
        raise ValueError(f"unknown tie_rule {tie_rule}")
    assign, prices, stats, status = fn(cost.detach(), sched, int(max_iter), int(path), int(tie_rule))
    if check:
        st = int(status.item())
        _lib.check(st, "auction kernel")
    if squeeze:
        assign, prices, stats = assign[0], prices[0], stats[0]
    return (assign, prices, stats, status) if return_status else (assign, prices, stats)


class AuctionB200:
    """Backend plug-in with the reference backend's interface.

    ``AuctionB200(epsilon, max_iter).solve(cost) -> (assignment, prices)``:
    assignment (B,N) int64, -1 for rows left unassigned after max_iter rounds;
    prices (B,M) fp32 (fp64 for fp64 input).  Same constructor and return
    contract as AuctionTorch (torch_backend.py:4-9,158).
    """

    def __init__(self, epsilon: EpsArg = 1e-2, max_iter: int = 1000, path: int = _lib.PATH_AUTO,
                 tie_rule: int = _lib.TIE_HIGHEST_ROW):
        self.epsilon = epsilon
        self.max_iter = max_iter
        self.path = path
        self.tie_rule = tie_rule
        self.last_stats = None

    def solve(self, cost_matrix: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Solve on the GPU.  A cost in host memory (the reference's backends
        accept CPU tensors) is copied to the current CUDA device, solved there
        by the same kernels, and the results are copied back to its device;
        without a CUDA device this raises (there is no CPU solver)."""
        if not cost_matrix.is_cuda:
            dev = _staging_device()
            assign, prices = self.solve(cost_matrix.to(dev))
            return assign.to(cost_matrix.device), prices.to(cost_matrix.device)
        assign, prices, stats = solve(cost_matrix, self.epsilon, self.max_iter, self.path, tie_rule=self.tie_rule)
        self.last_stats = stats
        return assign, prices


def _staging_device() -> torch.device:
    """The CUDA device a host-memory cost is solved on (the current one)."""
    if not torch.cuda.is_available():
        raise RuntimeError("the B200 auction solver needs a CUDA device; none is visible "
                           "(there is no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())
