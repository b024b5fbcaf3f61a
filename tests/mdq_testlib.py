"""Helpers shared by the tests: state construction and the reference extension.

The reference extension (``oracle/_ref/stquant_timetest_cpp*.so``) is the
reference's own kernel built from its sources by ``oracle/build_ref.py``; it
is used here only as the checker.
"""
from __future__ import annotations

import glob
import importlib
import importlib.machinery
import importlib.util
import os
import sys

import numpy as np
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(REPO, "oracle", "_ref")

CODE_DTYPES = {
    "packed4": (torch.uint8, None),
    "s8u8": (torch.int8, torch.uint8),
    "s16u16": (torch.int16, torch.uint16),
    "s32u32": (torch.int32, torch.uint32),
}


_REF_EXT = None
_REF_CLASSES = None


def load_reference_kernel():
    """The reference's compiled extension from oracle/_ref (GPU box), loaded
    from its file under its own module name (this repository's drop-in shim
    of the same name, stream-mm2026_b200/stquant_timetest_cpp.py, may be on
    sys.path too; it is never what this returns)."""
    global _REF_EXT
    if _REF_EXT is None:
        found = glob.glob(os.path.join(REF_DIR, "stquant_timetest_cpp*.so"))
        if not found:
            raise RuntimeError("oracle/_ref has no reference build; run python oracle/build_ref.py")
        import torch  # noqa: F401  (the extension links against torch)

        loader = importlib.machinery.ExtensionFileLoader("stquant_timetest_cpp", found[0])
        spec = importlib.util.spec_from_file_location("stquant_timetest_cpp", found[0],
                                                      loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _REF_EXT = mod
    return _REF_EXT


def load_reference_classes():
    """The reference's own optimizer classes, unmodified
    (CUDA/stquant_opt_simple.py:MDQAdamWSimple and
    CUDA/stquant_opt_fused_io.py:MDQAdamWSimpleFusedIO, byte-compiled into
    oracle/_ref by oracle/build_ref.py), bound to the reference's own compiled
    kernel.  Returns (MDQAdamWSimple, MDQAdamWSimpleFusedIO)."""
    global _REF_CLASSES
    if _REF_CLASSES is None:
        from oracle import build_ref

        ext = load_reference_kernel()
        simple = build_ref.load_python_module("stquant_opt_simple",
                                              {"stquant_timetest_cpp": ext})
        fused = build_ref.load_python_module("stquant_opt_fused_io",
                                             {"stquant_timetest_cpp": ext,
                                              "stquant_opt_simple": simple})
        for name in ("stquant_opt_simple", "stquant_opt_fused_io"):
            sys.modules.pop(name, None)
        _REF_CLASSES = (simple.MDQAdamWSimple, fused.MDQAdamWSimpleFusedIO)
    return _REF_CLASSES


class State:
    """One tensor's parameters, codes and block scales (reference layout)."""

    def __init__(self, n, block, layout, device, seed=0):
        g = torch.Generator().manual_seed(seed)
        self.n, self.block, self.layout = n, block, layout
        nb = (n + block - 1) // block
        self.p = (torch.randn(n, generator=g) * 0.02).to(device)
        mdt, vdt = CODE_DTYPES[layout]
        self.m = torch.zeros(n, dtype=mdt, device=device)
        if layout == "packed4":
            self.m.fill_(8)  # code pair (0, 0)
            self.v = torch.empty(0, dtype=torch.uint8, device=device)
        else:
            self.v = torch.zeros(n, dtype=vdt, device=device)
        self.sm = torch.zeros(nb, device=device)
        self.sv = torch.zeros(nb, device=device)
        self.vmin = torch.full((nb,), -20.0, device=device)

    def clone(self):
        o = State.__new__(State)
        o.n, o.block, o.layout = self.n, self.block, self.layout
        for k in ("p", "m", "v", "sm", "sv", "vmin"):
            setattr(o, k, getattr(self, k).clone())
        return o

    def tensors(self):
        return self.p, self.m, self.v, self.sm, self.sv, self.vmin

    def mismatches(self, other) -> dict:
        out = {}
        for k in ("p", "m", "v", "sm", "sv", "vmin"):
            a, b = getattr(self, k), getattr(other, k)
            if a.numel() == 0:
                out[k] = 0
                continue
            ai = a.view(torch.int32) if a.dtype == torch.float32 else a.to(torch.int64)
            bi = b.view(torch.int32) if b.dtype == torch.float32 else b.to(torch.int64)
            out[k] = int((ai != bi).sum())
        return out


def grads(n, steps, device, dtype=torch.float32, seed=1, scale=1e-3):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(n, generator=g) * scale).to(dtype).to(device) for _ in range(steps)]


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()
