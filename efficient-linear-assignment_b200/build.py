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
