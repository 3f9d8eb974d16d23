"""Seeded synthetic cost matrices for the benchmark configurations.

All inputs are drawn on the CPU with ``torch.Generator().manual_seed(seed)`` so
that the CPU oracle and the GPU see identical bits on any machine with the same
torch build; callers move them to the device afterwards.  The reference
publishes no dataset for this path; these generators follow the five
configurations its benchmark is quoted on (uniform costs, low-rank + noise
costs, integer costs with zero rows and constant columns).
"""
from __future__ import annotations

import torch


def cfg1(seed: int = 0) -> torch.Tensor:
    """B=4, N=M=128, fp32 uniform[0,1)."""
    g = torch.Generator().manual_seed(seed)
    return torch.rand(4, 128, 128, generator=g)


def uniform(B: int, N: int, M: int | None = None, seed: int = 1, dtype=torch.float32) -> torch.Tensor:
    """B x N x M uniform[0,1) fp32 costs, cast to ``dtype`` afterwards."""
    g = torch.Generator().manual_seed(seed)
    return torch.rand(B, N, M if M is not None else N, generator=g).to(dtype)


def cfg2(seed: int = 1) -> torch.Tensor:
    """B=1, N=M=4096, fp32 uniform[0,1)."""
    return uniform(1, 4096, 4096, seed)


def cfg3(dtype: torch.dtype, seed: int = 2) -> torch.Tensor:
    """B=1, N=M=4096, uniform[0,1) drawn in fp32 and cast to fp16/bf16."""
    return uniform(1, 4096, 4096, seed, dtype)


def cfg4(B: int = 256, N: int = 512, rank: int = 16, seed: int = 3) -> torch.Tensor:
    """Low-rank + noise costs: 0.5*minmax(U V^T) + 0.5*uniform, fp32.

    Draw order: U (B,N,r), V (B,N,r), then the (B,N,N) noise.
    """
    g = torch.Generator().manual_seed(seed)
    U = torch.randn(B, N, rank, generator=g)
    V = torch.randn(B, N, rank, generator=g)
    S = U @ V.transpose(1, 2)
    mn = S.amin(dim=(1, 2), keepdim=True)
    mx = S.amax(dim=(1, 2), keepdim=True)
    S = (S - mn) / (mx - mn)
    return 0.5 * S + 0.5 * torch.rand(B, N, N, generator=g)


def cfg5(B: int = 8, N: int = 8192, seed: int = 4) -> torch.Tensor:
    """Integer costs in {0..15} as bf16 (exact), 5% zero rows, 5% constant columns.

    Draw order: the (B,N,N) integers, then per problem: the zero-row
    permutation, the constant-column permutation and the constant.
    """
    g = torch.Generator().manual_seed(seed)
    C = torch.randint(0, 16, (B, N, N), generator=g, dtype=torch.int16).to(torch.bfloat16)
    k = int(0.05 * N)
    for b in range(B):
        r = torch.randperm(N, generator=g)[:k]
        C[b, r, :] = 0
        c = torch.randperm(N, generator=g)[:k]
        C[b, :, c] = torch.randint(0, 16, (1,), generator=g).to(torch.bfloat16)
    return C


def eps_schedule(eps0: float, eps_final: float, factor: float) -> list[float]:
    """eps0, eps0*factor, ... while above eps_final, then eps_final."""
    out, e = [], float(eps0)
    while e > eps_final:
        out.append(e)
        e *= factor
    out.append(float(eps_final))
    return out


CFG2_SCHEDULE = eps_schedule(1.0, 1e-2, 0.25)  # [1, .25, .0625, .015625, .01]
