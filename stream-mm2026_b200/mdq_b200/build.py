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
import tempfile
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(PKG_DIR)                 # stream-mm2026_b200/
REPO_ROOT = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO_ROOT, "include")
LIB_PATH = os.path.join(PKG_DIR, "libmdq.so")

SOURCES = ["mdq_step.cu", "mdq_stats.cu", "mdq_tiles_packed4.cu", "mdq_tiles_s8u8.cu",
           "mdq_tiles_s16u16.cu", "mdq_tiles_s32u32.cu", "mdq_tiles_m8v4.cu",
           "mdq_blocks_packed4.cu", "mdq_blocks_s8u8.cu", "mdq_blocks_s16u16.cu",
           "mdq_blocks_s32u32.cu", "mdq_blocks_m8v4.cu", "mdq_staged_s8u8.cu", "mdq_staged_packed4.cu",
           "mdq_fakequant.cu"]
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
    """Build libmdq.so unless it is newer than every source; return its path.

    Each translation unit compiles in its own nvcc process (in parallel),
    then one nvcc call links the shared library."""
    if not force and up_to_date():
        return LIB_PATH
    common = [nvcc(), *GENCODE, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              f"-I{INCLUDE}", f"-I{CSRC}"]
    if verbose:
        common.insert(1, "-Xptxas=-v")
    with tempfile.TemporaryDirectory(prefix="mdq_build_") as tmpdir:
        objs = [os.path.join(tmpdir, os.path.splitext(src)[0] + ".o") for src in SOURCES]

        def compile_one(i: int) -> None:
            cmd = [*common, "-c", os.path.join(CSRC, SOURCES[i]), "-o", objs[i]]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)

        workers = max(1, min(len(SOURCES), os.cpu_count() or 1))
        with ThreadPoolExecutor(max_workers=workers) as pool:
            list(pool.map(compile_one, range(len(SOURCES))))
        tmp = LIB_PATH + ".tmp"
        subprocess.run([nvcc(), *GENCODE, "-shared", "-o", tmp, *objs], check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
