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

The reference's pure-PyTorch optimizer (``baseline/mdqbock_newhook.py``) and
its two CUDA optimizer classes (``CUDA/stquant_opt_simple.py``,
``CUDA/stquant_opt_fused_io.py``) are byte-compiled the same way: each is
compiled where it lies into sourceless bytecode ``oracle/_ref/<module>.pycode``
(same interpreter as the GPU box; the suffix is not ``.pyc`` so that tools
which drop Python caches keep it), so the GPU box, which has no reference
checkout, can load and run the reference's own unmodified classes beside ours
(the timed CPU baseline of ``bench.py --impl reference`` and the GPU parity
tests) with ``load_python_module``.

The checkout is found from ``--reference``, else ``MDQ_REFERENCE_ROOT``, else
the ``reference_path`` that ``BASELINE.json`` records.

Usage:  python oracle/build_ref.py [--reference PATH]
"""
from __future__ import annotations

import argparse
import json
import os
import py_compile
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
MODULE = "stquant_timetest_cpp"


REPO = os.path.dirname(HERE)
# (module name, path within the reference checkout)
PY_MODULES = (("mdqbock_newhook", os.path.join("baseline", "mdqbock_newhook.py")),
              ("stquant_opt_simple", os.path.join("CUDA", "stquant_opt_simple.py")),
              ("stquant_opt_fused_io", os.path.join("CUDA", "stquant_opt_fused_io.py")))


def reference_root(explicit: str | None = None) -> str | None:
    """The reference checkout: explicit argument, MDQ_REFERENCE_ROOT, or
    BASELINE.json's ``reference_path``; None when none of them exists."""
    cands = [explicit, os.environ.get("MDQ_REFERENCE_ROOT")]
    try:
        with open(os.path.join(REPO, "BASELINE.json")) as f:
            cands.append(json.load(f).get("reference_path"))
    except (OSError, ValueError):
        pass
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "CUDA")):
            return c
    return None


BYTECODE_SUFFIX = ".pycode"


def python_modules_built() -> bool:
    return all(os.path.isfile(os.path.join(OUT_DIR, m + BYTECODE_SUFFIX)) for m, _ in PY_MODULES)


def load_python_module(name: str, extra_modules: dict | None = None):
    """Load the reference module `name` from its bytecode in oracle/_ref and
    return it (registered in sys.modules under `name`).  `extra_modules`
    (name -> module) are visible in sys.modules while it executes, so its own
    imports resolve to the reference's files; they are removed afterwards
    unless they were there before."""
    import importlib.machinery
    import importlib.util

    path = os.path.join(OUT_DIR, name + BYTECODE_SUFFIX)
    if not os.path.isfile(path):
        raise FileNotFoundError(f"{path}: run python oracle/build_ref.py")
    extra = dict(extra_modules or {})
    saved = {k: sys.modules.get(k) for k in extra}
    try:
        sys.modules.update(extra)
        loader = importlib.machinery.SourcelessFileLoader(name, path)
        spec = importlib.util.spec_from_file_location(name, path, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        loader.exec_module(mod)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return mod


def stage_python(reference_root: str) -> list[str]:
    """Byte-compile the reference's optimizer modules into oracle/_ref."""
    os.makedirs(OUT_DIR, exist_ok=True)
    out = []
    for mod, rel in PY_MODULES:
        src = os.path.join(reference_root, rel)
        dst = os.path.join(OUT_DIR, mod + BYTECODE_SUFFIX)
        py_compile.compile(src, cfile=dst, doraise=True,
                           invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
        out.append(dst)
    return out


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
    stage_python(reference_root)
    return path


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="reference checkout (default: MDQ_REFERENCE_ROOT, else BASELINE.json)")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    root = reference_root(a.reference)
    if root is None:
        ap.error("reference checkout not found: pass --reference or set MDQ_REFERENCE_ROOT")
    print(build(root, a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
