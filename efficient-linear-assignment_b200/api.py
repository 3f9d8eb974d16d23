"""Public API: ``linear_assignment`` and its IMLE autograd, as in the reference.

Mirrors src/efficient_linear_assignment/auction/api.py of the reference:
same signature, shape check (N and M multiples of 8, ValueError otherwise),
(B,N) int64 indices with unassigned rows reported as column 0 (the argmax of an
all-zero one-hot row, api.py:64-71,174), or the differentiable (B,N,M) one-hot
whose backward re-solves on ``C + lambda*G`` with lambda = 1 (api.py:82-149).
"""
from __future__ import annotations

from typing import Sequence, Union

import torch

from .solver import AuctionB200

# Backend registry (api.py:7-47).  Every name runs the B200 solver; 'torch'
# is accepted because the results are those of the reference's torch backend.
BACKENDS = {
    "b200": AuctionB200,
    "cuda": AuctionB200,
    "cpp": AuctionB200,
    "torch": AuctionB200,
}


def _one_hot(assignment: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """(B,N) columns -> (B,N,M) one-hot in like.dtype; rows at -1 stay zero."""
    P = torch.zeros_like(like)
    valid = assignment >= 0
    P.scatter_(2, assignment.clamp(min=0).unsqueeze(2), valid.unsqueeze(2).to(like.dtype))
    return P


def _solver(backend_name: str, epsilon, max_iter: int):
    if backend_name not in BACKENDS:
        raise ValueError(f"Backend '{backend_name}' not available. Options: {list(BACKENDS.keys())}")
    return BACKENDS[backend_name](epsilon=epsilon, max_iter=max_iter)


def _scatter_rows(out: torch.Tensor, assignment: torch.Tensor, value: float) -> None:
    """out[b, i, assignment[b, i]] += value for every assigned row (-1 rows skipped)."""
    valid = (assignment >= 0).unsqueeze(2).to(out.dtype)
    out.scatter_add_(2, assignment.clamp(min=0).unsqueeze(2), valid * value)


class AuctionIMLE(torch.autograd.Function):
    """Forward: hard assignment as a one-hot.  Backward: IMLE difference
    ``P(C + lambda*G) - P(C)`` divided by lambda (reference api.py:49-149).
    The target solve reads ``C`` and ``G`` and forms ``C + lambda*G`` in the
    kernel's loads (no dense target tensor) wherever the one-CTA or grid kernel
    runs the size; otherwise it solves the built sum.

    Only the (B,N) assignment is saved, not the dense forward one-hot, and the
    gradient is built as one zero fill plus two sparse row scatters (+1/lambda
    at the target column, -1/lambda at the forward column); the values equal
    the reference's dense ``(P_target - P_forward) / lambda``.
    """

    @staticmethod
    def forward(ctx, cost_matrix, epsilon, max_iter, backend_name):
        solver = _solver(backend_name, epsilon, max_iter)
        assignment, _ = solver.solve(cost_matrix)
        P = _one_hot(assignment, cost_matrix)
        ctx.save_for_backward(cost_matrix, assignment)
        ctx.epsilon = epsilon
        ctx.max_iter = max_iter
        ctx.backend_name = backend_name
        ctx.imle_lambda = 1.0
        return P

    @staticmethod
    def backward(ctx, grad_output):
        cost_matrix, assignment_f = ctx.saved_tensors
        lam = ctx.imle_lambda
        solver = _solver(ctx.backend_name, ctx.epsilon, ctx.max_iter)
        assignment_t = None
        if isinstance(solver, AuctionB200) and grad_output.shape == cost_matrix.shape \
                and grad_output.dtype == cost_matrix.dtype and cost_matrix.is_cuda and grad_output.is_cuda:
            # the target cost C + lam*G is read from the two tensors by the
            # kernel (ela_auction_solve_sum), not built (reference api.py:106-111)
            from .solver import _as_schedule, auction_solve_sum
            from . import _lib
            try:
                a, _, _, status = auction_solve_sum(cost_matrix.detach(), grad_output.detach(), lam,
                                                    _as_schedule(ctx.epsilon), int(ctx.max_iter), solver.path,
                                                    solver.tie_rule)
                _lib.check(int(status.item()), "auction kernel")
                assignment_t = a
            except _lib.AuctionError as e:
                if e.status != _lib.ELA_ERR_UNSUPPORTED:
                    raise
        if assignment_t is None:  # sizes only the cluster kernel runs: solve the built sum
            assignment_t, _ = solver.solve(cost_matrix + lam * grad_output)
        grad = torch.zeros_like(cost_matrix)
        _scatter_rows(grad, assignment_t, 1.0 / lam)
        _scatter_rows(grad, assignment_f, -1.0 / lam)
        return grad, None, None, None


def linear_assignment(cost_matrix: torch.Tensor, epsilon: Union[float, Sequence[float]] = 1e-2,
                      max_iter: int = 1000, backend: str = "b200", return_indices: bool = True,
                      auto_pad: bool = False):
    """Solve the linear assignment problem (minimise total cost) by auction.

    cost_matrix: (B,N,M) or (N,M) tensor, fp32/fp16/bf16/fp64, N and M
    multiples of 8 (as in the reference) unless auto_pad.  A CUDA tensor is
    solved on its device; a host tensor (which the reference's backends also
    take) is copied to the current CUDA device, solved there, and the result
    comes back on the host.  There is no CPU solver: without a GPU this raises.  epsilon: constant
    epsilon (the reference's only mode) or an epsilon-scaling schedule.
    Returns (B,N) int64 indices when return_indices, else the differentiable
    (B,N,M) one-hot.

    auto_pad=True accepts any N and M and returns what solving
    ``pad_input(cost)`` and keeping the real rows (``unpad_result``) returns.
    When M needs padding, M >= 128 and there are no more dummy rows than
    dummy columns, the problem is solved as given, without the copy: the
    dummy columns (cost 1e9 for real rows) never enter a real row's top-2 bid
    nor its tie choice (for rows of 128 or more columns torch.topk's tied
    column is fixed by the first two occurrences of the maximum), and the
    dummy rows (cost 0 on dummy columns, 1e9 on real ones) settle on dummy
    columns, so the real rows' rounds are the same.  Below 128 columns the
    tied column comes from an introselect over the whole row, whose steps
    depend on the row length, and with more dummy rows than dummy columns the
    dummy rows bid on real columns: both solve the padded problem, whose
    padding the kernel synthesises in its loaders (``ela_auction_solve_padded``),
    so no padded copy is built for indices either.
    """
    is_batched = cost_matrix.ndim == 3
    if not is_batched:
        cost_matrix = cost_matrix.unsqueeze(0)
    _, N, M = cost_matrix.shape
    if auto_pad and (N % 8 != 0 or M % 8 != 0):
        from .utils import get_pad_size
        pn, pm = get_pad_size(N), get_pad_size(M)
        if pm == 0 or pn > pm or M < 128:
            # the padding could change a bid or a tie: solve the padded problem,
            # its padding synthesised by the kernel (no padded copy)
            if return_indices:
                if backend not in BACKENDS:
                    raise ValueError(f"Backend '{backend}' not available. Options: {list(BACKENDS.keys())}")
                from .solver import _as_schedule, _staging_device, auction_solve_padded
                from . import _lib
                src = cost_matrix.detach()
                on_host = not src.is_cuda
                if on_host:  # host memory: solved on the current CUDA device, indices copied back
                    src = src.to(_staging_device())
                assign, _, _, status = auction_solve_padded(src, _as_schedule(epsilon), int(max_iter))
                _lib.check(int(status.item()), "auction kernel")
                idx = assign[:, :N].clamp(min=0)
                if on_host:
                    idx = idx.to(cost_matrix.device)
                return idx if is_batched else idx.squeeze(0)
            from .utils import pad_input  # differentiable one-hot: autograd needs the padded tensor
            padded, _ = pad_input(cost_matrix)
            out = linear_assignment(padded, epsilon, max_iter, backend, False)[:, :N, :M]
            return out if is_batched else out.squeeze(0)
    elif N % 8 != 0 or M % 8 != 0:
        raise ValueError(f"Input dimensions must be multiples of 8. Got shape {cost_matrix.shape}. "
                         "Please pad your input.")
    if return_indices:
        solver = _solver(backend, epsilon, max_iter)
        assignment, _ = solver.solve(cost_matrix.detach())
        idx = assignment.clamp(min=0)
        return idx if is_batched else idx.squeeze(0)
    P = AuctionIMLE.apply(cost_matrix, epsilon, max_iter, backend)
    return P if is_batched else P.squeeze(0)
