"""B200-native auction solver for the linear assignment problem.

Drop-in for ``efficient_linear_assignment.linear_assignment`` (auction path):
hand-written sm_100a CUDA kernels behind a C ABI (include/ela_auction.h).
"""
from .api import BACKENDS, AuctionIMLE, linear_assignment
from .solver import AuctionB200, auction_solve, auction_solve_op, auction_solve_padded, auction_solve_sum, compute_bids, implicit_costs, solve, solve_implicit
from ._lib import AuctionError, PATH_AUTO, PATH_CTA, PATH_GRID, PATH_CLUSTER, TIE_HIGHEST_ROW, TIE_LOWEST_ROW
from . import workloads
from .utils import get_pad_size, pad_input, pad_to_shape, unpad_result

__all__ = ["linear_assignment", "AuctionIMLE", "AuctionB200", "BACKENDS", "solve",
           "auction_solve", "auction_solve_op", "auction_solve_padded", "auction_solve_sum", "compute_bids", "solve_implicit", "implicit_costs", "AuctionError", "PATH_AUTO", "PATH_CTA", "PATH_GRID", "PATH_CLUSTER",
           "TIE_HIGHEST_ROW", "TIE_LOWEST_ROW", "workloads",
           "get_pad_size", "pad_input", "pad_to_shape", "unpad_result"]
