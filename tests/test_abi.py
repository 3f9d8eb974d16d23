"""CPU tests of the C ABI library: it builds, loads and exports every symbol
include/ela_auction.h declares (no compute calls: there is no GPU here)."""
import ctypes
import os
import re

import pytest

import efficient_linear_assignment_b200 as ela
from efficient_linear_assignment_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"\b(ela_\w+)\s*\(", src)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert "ela_auction_solve" in names
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_status_strings_and_version():
    assert _lib.load().ela_auction_version() >= 200
    assert _lib.status_string(0) == "ok"
    assert "timed out" in _lib.status_string(3)


def test_solve_rejects_bad_arguments_without_touching_the_gpu():
    lib = _lib.load()
    eps = (ctypes.c_double * 1)(1e-2)
    null = ctypes.c_void_p(0)
    # bad dtype
    assert lib.ela_auction_solve(null, 9, 1, 8, 8, 64, 8, eps, 1, 10, 0, 0, null, null, null, null, null, 0, null) == 1
    # epsilon must be > 0
    bad = (ctypes.c_double * 1)(0.0)
    assert lib.ela_auction_solve(null, 0, 1, 8, 8, 64, 8, bad, 1, 10, 0, 0, null, null, null, null, null, 0, null) == 1
    # unknown tie rule (checked before any device work)
    one = ctypes.c_void_p(256)
    assert lib.ela_auction_solve(one, 0, 1, 8, 8, 64, 8, eps, 1, 10, 0, 7, one, one, null, null, one, 1 << 20,
                                 null) == 1
    assert lib.ela_auction_solve_noalloc(one, 0, 1, 8, 8, 64, 8, eps, 1, 10, 0, 7, one, one, null, null, null) == 1
    # empty batch is a no-op
    assert lib.ela_auction_solve(null, 0, 0, 8, 8, 64, 8, eps, 1, 10, 0, 0, null, null, null, null, null, 0, null) == 0


def test_torch_operator_library_loads_and_registers():
    """The C++ operator over the C ABI (csrc/ela_torch_op.cpp) loads without a
    GPU and registers torch.ops.ela_native.auction_solve."""
    import torch
    from efficient_linear_assignment_b200 import solver
    op = solver._native_op()
    assert op is torch.ops.ela_native.auction_solve
    with pytest.raises(RuntimeError, match="CUDA"):
        ela.auction_solve(torch.rand(1, 8, 8), [1e-2], 10, 0)
