"""Generate host-logic golden trajectories from the reference's optimizer classes.

Run in a container that holds the reference checkout (``--reference PATH``,
else ``MDQ_REFERENCE_ROOT``, else BASELINE.json's ``reference_path``).  The reference classes
(CUDA/stquant_opt_simple.py:MDQAdamWSimple, CUDA/stquant_opt_fused_io.py:
MDQAdamWSimpleFusedIO) import the CUDA extension ``stquant_timetest_cpp`` at
module top; here that module is provided by the CPU oracle
(oracle/oracle.py:fused_mdq_adamw_cpu, the reference binding's argument list),
so the reference's own host logic -- bit policy, state init, storage align /
pack, FusedIO step counting -- runs unmodified on CPU tensors.

Output: tests/golden/host_trajectories.npz, recording per step every
parameter's current_bit, step, storage dtypes and last_score, and at the end
the codes, scales and parameters.  tests/test_host_parity.py replays the same
scenario through mdq_b200's optimizer classes (with the same oracle kernel)
and requires identical records.
"""
from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "tests"))

from oracle import oracle  # noqa: E402
from host_scenario import SCENARIOS, run_scenario  # noqa: E402



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

def import_reference_classes(reference_root: str):
    fake = types.ModuleType("stquant_timetest_cpp")
    fake.fused_mdq_adamw = oracle.fused_mdq_adamw_cpu
    sys.modules["stquant_timetest_cpp"] = fake
    sys.path.insert(0, os.path.join(reference_root, "CUDA"))
    import stquant_opt_fused_io  # noqa: E402
    import stquant_opt_simple  # noqa: E402
    return stquant_opt_simple.MDQAdamWSimple, stquant_opt_fused_io.MDQAdamWSimpleFusedIO


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    ap.add_argument("--out", default=os.path.join(HERE, "host_trajectories.npz"))
    a = ap.parse_args()
    a.reference = _reference_root(a.reference)
    torch.set_num_threads(1)
    simple, fused = import_reference_classes(a.reference)
    classes = {"simple": simple, "fusedio": fused}
    out = {}
    for name, sc in SCENARIOS.items():
        rec = run_scenario(classes[sc["cls"]], sc)
        for k, v in rec.items():
            out[f"{name}/{k}"] = v
    np.savez_compressed(a.out, **out)
    print(a.out, sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main()
