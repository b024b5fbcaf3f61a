"""Our kernel against the committed golden vectors of the reference's kernel:
bit-identical codes, scales and parameters (exact parameter mode)."""
import os

import numpy as np
import pytest
import torch

from mdq_b200 import kernels

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "kernel_golden.npz")
HP = (0.9, 0.999, 1e-3, 0.01, 1e-8)


def test_kernel_reproduces_golden_vectors(cuda_device):
    g = np.load(GOLD)
    for case in sorted({k.split("/")[0] for k in g.files}):
        lay, bits, n, block = (int(x) for x in g[f"{case}/meta"])
        t = {k: torch.from_numpy(g[f"{case}/in_{k}"].copy()).to(cuda_device)
             for k in ("p", "m", "v", "sm", "sv", "vmin")}
        for s, grad in enumerate(g[f"{case}/grads"], start=1):
            kernels.fused_mdq_adamw(t["p"], torch.from_numpy(grad).to(cuda_device), t["m"], t["v"],
                                    t["sm"], t["sv"], t["vmin"], *HP, s, bits, block)
        torch.cuda.synchronize()
        for k in ("p", "m", "v", "sm", "sv", "vmin"):
            np.testing.assert_array_equal(t[k].cpu().numpy().view(np.uint8),
                                          g[f"{case}/out_{k}"].view(np.uint8), err_msg=f"{case} {k}")
