"""Golden vectors for robust_quantize from the reference's pure-PyTorch
optimizer (baseline/mdqbock_newhook.py:58-83, MDQAdamW.robust_quantize).

Run where the reference checkout exists (``--reference PATH``, else
``MDQ_REFERENCE_ROOT``, else BASELINE.json's ``reference_path``):

    python tests/golden/make_robust_quantize_golden.py [--reference PATH]

Writes tests/golden/robust_quantize.npz: seeded m-like and v-like tensors of
awkward sizes and their fake-quantised values for bits 4, 8, 16 (and 32,
which the reference returns unchanged) and block sizes 2048, 256, 100.
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))



def _reference_root(explicit):
    """The reference checkout (see oracle/build_ref.py:reference_root)."""
    repo = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    if repo not in sys.path:
        sys.path.insert(0, repo)
    from oracle.build_ref import reference_root

    root = reference_root(explicit)
    if root is None:
        raise SystemExit("reference checkout not found: pass --reference or set MDQ_REFERENCE_ROOT")
    return root

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    ap.add_argument("--out", default=os.path.join(HERE, "robust_quantize.npz"))
    a = ap.parse_args()
    a.reference = _reference_root(a.reference)
    sys.path.insert(0, os.path.join(a.reference, "baseline"))
    from mdqbock_newhook import MDQAdamW  # noqa: E402

    opt = MDQAdamW([torch.nn.Parameter(torch.zeros(1))])
    g = torch.Generator().manual_seed(0)
    out = {}
    for i, shape in enumerate([(5000,), (64, 65), (3,), (4096,)]):
        m = torch.randn(shape, generator=g) * 1e-3
        v = torch.rand(shape, generator=g) * 1e-6 + 1e-9
        out[f"t{i}/m"] = m.numpy()
        out[f"t{i}/v"] = v.numpy()
        for bits in (4, 8, 16, 32):
            for block in (2048, 256, 100):
                out[f"t{i}/m_b{bits}_k{block}"] = opt.robust_quantize(m, bits, False, block).numpy()
                out[f"t{i}/v_b{bits}_k{block}"] = opt.robust_quantize(v, bits, True, block).numpy()
    np.savez_compressed(a.out, **out)
    print(a.out)


if __name__ == "__main__":
    main()
