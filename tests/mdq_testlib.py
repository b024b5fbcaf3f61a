"""Helpers shared by the tests: state construction and the reference extension.

The reference extension (``oracle/_ref/stquant_timetest_cpp*.so``) is the
reference's own kernel built from its sources by ``oracle/build_ref.py``; it
is used here only as the checker.
"""
from __future__ import annotations

import glob
import importlib
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


def load_reference_kernel():
    """Import the reference's compiled extension from oracle/_ref (GPU box)."""
    if not glob.glob(os.path.join(REF_DIR, "stquant_timetest_cpp*.so")):
        raise RuntimeError("oracle/_ref has no reference build; run python oracle/build_ref.py")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    return importlib.import_module("stquant_timetest_cpp")


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
