"""Compile the sm_100a kernels into the in-tree shared library ``libmdq.so``.

The library is a plain C ABI (``include/mdq.h``) built with nvcc directly; it
links no torch symbols, so any host language can bind it.  The build writes
next to this file so the .so travels with the source tree.

    python -m mdq_b200.build            # from stream-mm2026_b200/
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(PKG_DIR)                 # stream-mm2026_b200/
REPO_ROOT = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO_ROOT, "include")
LIB_PATH = os.path.join(PKG_DIR, "libmdq.so")

SOURCES = ["mdq_step.cu", "mdq_stats.cu"]
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand) and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")
    return cand


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, s) for s in SOURCES]
    files += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    files.append(os.path.join(INCLUDE, "mdq.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Build libmdq.so unless it is newer than every source; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc(), *GENCODE, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-shared", f"-I{INCLUDE}", f"-I{CSRC}", "-o", tmp,
           *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
