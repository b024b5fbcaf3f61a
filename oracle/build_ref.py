"""Build the reference's own fused MDQ-AdamW CUDA extension from its sources.

TEST INFRASTRUCTURE ONLY.  The product never imports, links or executes
anything under ``oracle/``; only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may.

The reference ships its kernel as two source files,
``CUDA/stquant_kernel.cu`` and ``CUDA/stquant_core.cpp`` (module name
``stquant_timetest_cpp``, bound at ``CUDA/stquant_core.cpp:9-15``).  Its own
``CUDA/setup.py:15-17`` compiles them with ``-O3 -lineinfo`` and no explicit
arch.  This recipe compiles the same two files, where they lie in the read-only
reference checkout, with the same optimisation flags plus an explicit
``sm_100`` target, and writes every output into ``oracle/_ref/`` (git-ignored,
but it travels to the GPU box with the snapshot).  No reference source is
copied into this repository.

On the GPU box the resulting ``oracle/_ref/stquant_timetest_cpp*.so`` is the
bit-exact oracle for codes and block scales: the kernel under test is compared
against the reference's own arithmetic, CUDA libm included.

Usage:  python oracle/build_ref.py [--reference /path/to/reference]
"""
from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
MODULE = "stquant_timetest_cpp"


def built_module_path() -> str | None:
    """Path of the built reference extension, or None when it is absent."""
    if not os.path.isdir(OUT_DIR):
        return None
    for f in sorted(os.listdir(OUT_DIR)):
        if f.startswith(MODULE) and f.endswith(".so"):
            return os.path.join(OUT_DIR, f)
    return None


def build(reference_root: str, verbose: bool = False) -> str:
    """Compile the reference extension into oracle/_ref and return the .so path."""
    src_dir = os.path.join(reference_root, "CUDA")
    sources = [os.path.join(src_dir, "stquant_core.cpp"),
               os.path.join(src_dir, "stquant_kernel.cu")]
    for s in sources:
        if not os.path.isfile(s):
            raise FileNotFoundError(s)
    os.makedirs(OUT_DIR, exist_ok=True)
    from torch.utils.cpp_extension import load

    # Same flags as the reference build (setup.py: cxx -O3, nvcc -O3 -lineinfo);
    # the arch is the only addition, since the reference relies on
    # TORCH_CUDA_ARCH_LIST and ships no Blackwell target.
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    load(
        name=MODULE,
        sources=sources,
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "-lineinfo"],
        build_directory=OUT_DIR,
        verbose=verbose,
        is_python_module=True,
    )
    path = built_module_path()
    if path is None:
        raise RuntimeError("reference extension did not build")
    return path


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MDQ_REFERENCE_ROOT", "/root/reference"))
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.reference, a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
