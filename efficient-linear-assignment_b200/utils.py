"""Padding helpers with the reference's contract (src/efficient_linear_assignment/utils.py).

The reference requires N and M to be multiples of 8 (auction/api.py:164-166)
and offers pad_input/unpad_result to get there: real rows see cost 1e9 on the
dummy columns, dummy rows see 1e9 on the real columns and 0 on the dummy ones
(utils.py:32-105).  The same functions are provided here (device-side torch
ops, no host round trip).  The CUDA solver itself has no size restriction, so
``linear_assignment(..., auto_pad=True)`` solves an unpadded problem directly
instead of materialising the padded copy (see api.py).
"""
from __future__ import annotations

from typing import Tuple

import torch

PAD_COST = 1e9  # the reference's "large cost" for real<->dummy pairs (utils.py:83)


def get_pad_size(n: int, multiple: int = 8) -> int:
    """Amount to add to n to reach a multiple of `multiple` (utils.py:6-10)."""
    r = n % multiple
    return 0 if r == 0 else multiple - r


def pad_to_shape(tensor: torch.Tensor, target_shape: Tuple[int, ...], value: float = 0.0) -> torch.Tensor:
    """Pad the trailing end of every dimension up to target_shape (utils.py:12-30)."""
    pad = []
    for i in range(len(target_shape) - 1, -1, -1):
        pad.extend([0, target_shape[i] - tensor.shape[i]])
    return torch.nn.functional.pad(tensor, tuple(pad), value=value)


def pad_input(cost_matrix: torch.Tensor, multiple: int = 8) -> Tuple[torch.Tensor, Tuple[int, int, int]]:
    """Pad (B,N,M) costs so N and M are multiples of `multiple` (utils.py:32-105).

    Returns (padded, (B, N, M)).  Real/dummy blocks: real x real = cost,
    real x dummy = dummy x real = 1e9, dummy x dummy = 0 (only when both N and
    M are padded, as in the reference).
    """
    B, N, M = cost_matrix.shape
    pn, pm = get_pad_size(N, multiple), get_pad_size(M, multiple)
    if pn == 0 and pm == 0:
        return cost_matrix, (B, N, M)
    out = torch.full((B, N + pn, M + pm), PAD_COST, dtype=cost_matrix.dtype, device=cost_matrix.device)
    out[:, :N, :M] = cost_matrix
    if pn > 0 and pm > 0:
        out[:, N:, M:] = 0.0
    return out, (B, N, M)


def unpad_result(indices: torch.Tensor, original_shape: Tuple[int, int, int]) -> torch.Tensor:
    """Keep the rows of the original problem (utils.py:107-112)."""
    B, N, M = original_shape
    return indices[:, :N]
