"""Build the in-tree CUDA library libela_auction.so for sm_100a.

Run ``python efficient-linear-assignment_b200/build.py`` (or
``__graft_entry__.build()``).  nvcc cross-compiles, so no GPU is needed.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
SRC = os.path.join(PKG_DIR, "csrc", "ela_auction.cu")
OUT = os.path.join(PKG_DIR, "libela_auction.so")
INCLUDE = os.path.join(REPO_DIR, "include")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


OP_SRC = os.path.join(PKG_DIR, "csrc", "ela_torch_op.cpp")
OP_OUT = os.path.join(PKG_DIR, "libela_torch_op.so")


def build_op(force: bool = False) -> str:
    """Compile the C++ torch operator (torch.ops.ela_native.auction_solve) over
    libela_auction.so, unless it is newer than its sources."""
    deps = [OP_SRC, OUT, os.path.join(INCLUDE, "ela_auction.h")]
    if not force and os.path.exists(OP_OUT) and all(os.path.getmtime(OP_OUT) >= os.path.getmtime(d) for d in deps):
        return OP_OUT
    import torch
    tdir = os.path.dirname(torch.__file__)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "include")
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", os.path.join(tdir, "include"), "-I", os.path.join(tdir, "include", "torch", "csrc", "api", "include"),
           "-I", cuda_inc, "-I", INCLUDE, OP_SRC, "-o", OP_OUT + ".tmp", "-L", PKG_DIR, "-lela_auction",
           "-L", os.path.join(tdir, "lib"), "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
           "-Wl,-rpath,$ORIGIN"]
    subprocess.run(cmd, check=True)
    os.replace(OP_OUT + ".tmp", OP_OUT)
    return OP_OUT


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libela_auction.so unless it is newer than its sources."""
    deps = [SRC, os.path.join(PKG_DIR, "csrc", "ela_implicit.cuh"), os.path.join(INCLUDE, "ela_auction.h")]
    if not force and os.path.exists(OUT) and all(os.path.getmtime(OUT) >= os.path.getmtime(d) for d in deps):
        return OUT
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-o", OUT + ".tmp", SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_op(force="--force" in sys.argv))
