"""Golden vectors from the reference's own kernel (run on a GPU box).

Builds seeded states for every reference layout (packed4 / s8u8 / s16u16 /
s32u32), block sizes including a non-power-of-two one and a partial tail, and
runs three steps of the reference's compiled kernel
(``oracle/_ref/stquant_timetest_cpp``, built from CUDA/stquant_kernel.cu by
``oracle/build_ref.py``) with fp32 gradients.  Inputs and outputs go to
``tests/golden/kernel_golden.npz`` (a few hundred KB).

    python tests/golden/make_kernel_golden.py [--out PATH]
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from mdq_testlib import State, load_reference_kernel  # noqa: E402

CASES = [("packed4", 4, 5000, 256), ("packed4", 4, 4099, 1024), ("s8u8", 8, 3001, 128),
         ("s8u8", 4, 2500, 100), ("s16u16", 16, 2049, 512), ("s32u32", 32, 1500, 64)]
HP = (0.9, 0.999, 1e-3, 0.01, 1e-8)
STEPS = 3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "kernel_golden.npz"))
    a = ap.parse_args()
    ref = load_reference_kernel()
    dev = torch.device("cuda:0")
    out = {}
    for ci, (layout, bits, n, block) in enumerate(CASES):
        st = State(n, block, layout, dev, seed=ci)
        gen = torch.Generator().manual_seed(100 + ci)
        key = f"c{ci}"
        out[f"{key}/meta"] = np.array([["packed4", "s8u8", "s16u16", "s32u32"].index(layout),
                                       bits, n, block])
        for k in ("p", "m", "v", "sm", "sv", "vmin"):
            out[f"{key}/in_{k}"] = getattr(st, k).cpu().numpy().copy()
        grads = [(torch.randn(n, generator=gen) * 1e-3) for _ in range(STEPS)]
        out[f"{key}/grads"] = torch.stack(grads).numpy()
        prof = torch.empty(0, dtype=torch.int64, device=dev)
        for s, g in enumerate(grads, start=1):
            ref.fused_mdq_adamw(st.p, g.to(dev), st.m, st.v, st.sm, st.sv, st.vmin, *HP, s, bits,
                                block, prof)
        torch.cuda.synchronize()
        for k in ("p", "m", "v", "sm", "sv", "vmin"):
            out[f"{key}/out_{k}"] = getattr(st, k).cpu().numpy().copy()
    os.makedirs(os.path.dirname(a.out), exist_ok=True)
    np.savez_compressed(a.out, **out)
    print(a.out)


if __name__ == "__main__":
    main()
