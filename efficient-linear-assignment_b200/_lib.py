"""ctypes binding of libela_auction.so (the C ABI in include/ela_auction.h).

The library is required: importing the solver on a machine without it raises,
there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import OUT as LIB_PATH

ELA_OK = 0
ELA_ERR_ARGUMENT = 1
ELA_ERR_CUDA = 2
ELA_ERR_TIMEOUT = 3
ELA_ERR_UNSUPPORTED = 4
ELA_ERR_INTERNAL = 5

PATH_AUTO, PATH_CTA, PATH_GRID, PATH_CLUSTER = 0, 1, 2, 3
TIE_HIGHEST_ROW, TIE_LOWEST_ROW = 0, 1  # ELA_TIE_*: election rule among bids within 1e-5

# Every symbol include/ela_auction.h declares, with (restype, argtypes).
_c = ctypes
SIGNATURES = {
    "ela_auction_version": (_c.c_int, []),
    "ela_status_string": (_c.c_char_p, [_c.c_int]),
    "ela_auction_workspace_bytes": (_c.c_size_t, [_c.c_int, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int]),
    "ela_auction_solve": (_c.c_int, [
        _c.c_void_p, _c.c_int, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64,
        _c.POINTER(_c.c_double), _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_void_p, _c.c_void_p,
        _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t, _c.c_void_p]),
    "ela_auction_solve_noalloc": (_c.c_int, [
        _c.c_void_p, _c.c_int, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64,
        _c.POINTER(_c.c_double), _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_void_p, _c.c_void_p,
        _c.c_void_p, _c.c_void_p, _c.c_void_p]),
    "ela_auction_solve_padded": (_c.c_int, [
        _c.c_void_p, _c.c_int, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int,
        _c.POINTER(_c.c_double), _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_void_p, _c.c_void_p,
        _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t, _c.c_void_p]),
    "ela_auction_solve_sum": (_c.c_int, [
        _c.c_void_p, _c.c_void_p, _c.c_double, _c.c_int, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64,
        _c.c_int64, _c.POINTER(_c.c_double), _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_void_p, _c.c_void_p,
        _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t, _c.c_void_p]),
    "ela_auction_solve_implicit": (_c.c_int, [
        _c.c_void_p, _c.c_void_p, _c.c_int, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64,
        _c.POINTER(_c.c_double), _c.c_int, _c.c_int, _c.c_int, _c.c_void_p, _c.c_void_p, _c.c_void_p,
        _c.c_void_p, _c.c_void_p]),
    "ela_auction_implicit_costs": (_c.c_int, [
        _c.c_void_p, _c.c_void_p, _c.c_int, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_void_p,
        _c.c_void_p, _c.c_void_p]),
    "ela_auction_compute_bids": (_c.c_int, [
        _c.c_void_p, _c.c_int, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_void_p,
        _c.c_void_p, _c.c_double, _c.c_void_p, _c.c_void_p, _c.c_void_p]),
    "ela_auction_set_wait_limit_ns": (None, [_c.c_uint64]),
    "ela_auction_debug_skip_arrive": (None, [_c.c_int]),
}

_lib = None
_lock = threading.Lock()


class AuctionError(RuntimeError):
    """A status other than ELA_OK from the CUDA library."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {status_string(status)} (status {status})")


def load() -> ctypes.CDLL:
    """Load the library, raising if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                        "(no CPU fallback exists for this solver)")
                lib = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().ela_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != ELA_OK:
        raise AuctionError(status, where)
