"""Reference-written checkpoints and their continuations, for resume parity.

The reference's optimizer classes (CUDA/stquant_opt_simple.py, CUDA/
stquant_opt_fused_io.py; kernel supplied by the CPU oracle exactly as in
make_host_golden.py) run SAVE_AT steps of the host scenario; the parameters
and ``optimizer.state_dict()`` are written with torch.save, as the
reference's training script checkpoints (baseline/pretrain_gpt.py:321-332).
The reference run then continues for MORE steps, and its final parameters,
codes, scales, bit widths and step counters are recorded.

    python tests/golden/make_checkpoint_golden.py [--reference PATH]

Writes tests/golden/ref_ckpt_<cls>.pt and ref_ckpt_<cls>_final.npz.
tests/test_optimizer_api.py loads each checkpoint into mdq_b200's class of the
same name, continues, and requires the reference's final state bit for bit.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_host_golden import import_reference_classes  # noqa: E402
from host_scenario import SIZES, grads_for_step, make_params  # noqa: E402

SAVE_AT, MORE = 9, 7
KW = dict(lr=1e-3, weight_decay=0.01, layer_count=12, batch_size=16, update_freq=4,
          block_size=256)



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

def groups(params):
    half = (len(params) + 1) // 2
    return [{"params": params[:half]}, {"params": params[half:], "weight_decay": 0.0}]


def run(cls, params, opt, steps):
    for t in steps:
        for p, g in zip(params, grads_for_step(SIZES, t)):
            p.grad = g.clone()
        opt.step()


def final_record(params, opt):
    rec = {"total_steps": np.array(opt.total_steps)}
    for i, p in enumerate(params):
        st = opt.state[p]
        rec[f"p{i}"] = p.detach().numpy().copy()
        rec[f"bits{i}"] = np.array(int(st["current_bit"]))
        rec[f"step{i}"] = np.array(int(st["step"]))
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            t = st[k]
            rec[f"{k}{i}"] = t.view(torch.uint8).numpy().copy() if t.numel() else np.zeros(0, np.uint8)
            rec[f"{k}{i}_dtype"] = np.array(str(t.dtype))
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    a = ap.parse_args()
    a.reference = _reference_root(a.reference)
    torch.set_num_threads(1)
    simple, fused = import_reference_classes(a.reference)
    for name, cls in (("simple", simple), ("fusedio", fused)):
        params = make_params(SIZES)
        opt = cls(groups(params), **KW)
        run(cls, params, opt, range(1, SAVE_AT + 1))
        torch.save({"params": [p.detach().clone() for p in params], "optimizer": opt.state_dict()},
                   os.path.join(HERE, f"ref_ckpt_{name}.pt"))
        run(cls, params, opt, range(SAVE_AT + 1, SAVE_AT + MORE + 1))
        np.savez_compressed(os.path.join(HERE, f"ref_ckpt_{name}_final.npz"),
                            **final_record(params, opt))
        print(name, "bits", sorted({int(opt.state[p]["current_bit"]) for p in params}))


if __name__ == "__main__":
    main()
