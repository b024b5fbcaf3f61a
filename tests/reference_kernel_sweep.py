"""Time the reference's own fused kernel beside ours on the BASELINE config-2
points (test infrastructure: it runs the reference kernel that
oracle/build_ref.py built into oracle/_ref).

    python tests/reference_kernel_sweep.py [--out gpurun_out/reference_kernel_sweep.json]

For each point (4 / 8-bit codes, block 128 and 2048, which the reference's
CUDA path clamps to 1024; 2^20 ... 2^30 elements), both kernels take the same
fp32 gradients (the reference accepts no other dtype) and run 3 warm-up and 10
timed steps, CUDA events on the current stream.  Ours runs in both parameter
modes.  Prints one table row per point and writes the rows as JSON.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for _p in (os.path.join(REPO, "stream-mm2026_b200"), REPO, HERE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from mdq_b200 import kernels  # noqa: E402
from mdq_b200.kernels import LAYOUT_PACKED4, LAYOUT_S8U8, P_EXACT, P_FAST, StepItem  # noqa: E402
from mdq_testlib import State, load_reference_kernel  # noqa: E402


def timed(fn, steps=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(REPO, "gpurun_out", "reference_kernel_sweep.json"))
    a = ap.parse_args()
    dev = torch.device("cuda:0")
    ref = load_reference_kernel()
    rows = []
    print("| bits | block (quantised) | elements | reference ms | ours fast ms | ours exact ms "
          "| reference Gparams/s | ours fast Gparams/s | speed-up fast / exact |")
    for bits in (4, 8):
        layout = "packed4" if bits == 4 else "s8u8"
        lid = LAYOUT_PACKED4 if bits == 4 else LAYOUT_S8U8
        for block in (128, 2048):
            qb = min(block, 1024)
            for lg in (20, 24, 27, 30):
                n = 1 << lg
                st = State(n, qb, layout, dev)
                g = torch.randn(n, device=dev) * 1e-3
                prof = torch.empty(0, dtype=torch.int64, device=dev)
                t_ref = timed(lambda: ref.fused_mdq_adamw(st.p, g, st.m, st.v, st.sm, st.sv,
                                                          st.vmin, 0.9, 0.999, 1e-3, 0.01, 1e-8,
                                                          5, bits, block, prof))
                it = StepItem(p=st.p, grad=g, exp_avg=st.m,
                              exp_avg_sq=st.v if st.v.numel() else None, scale_m=st.sm,
                              scale_v=st.sv, v_min=st.vmin, step=5, block=qb, lr=1e-3,
                              weight_decay=0.01, eps=1e-8, beta1=0.9, beta2=0.999, m_bits=bits,
                              v_bits=bits, layout=lid)
                t_fast = timed(lambda: kernels.step_multi([it], p_mode=P_FAST))
                t_exact = timed(lambda: kernels.step_multi([it], p_mode=P_EXACT))
                gp = lambda t: n / t / 1e6  # noqa: E731
                row = dict(bits=bits, block=block, quant_block=qb, log2_elements=lg,
                           ref_ms=t_ref, fast_ms=t_fast, exact_ms=t_exact)
                rows.append(row)
                print(f"| {bits} | {block} ({qb}) | 2^{lg} | {t_ref:.4f} | {t_fast:.4f} | "
                      f"{t_exact:.4f} | {gp(t_ref):.1f} | {gp(t_fast):.1f} | "
                      f"{t_ref / t_fast:.1f}x / {t_ref / t_exact:.1f}x |", flush=True)
                del st, g
                torch.cuda.empty_cache()
    os.makedirs(os.path.dirname(a.out), exist_ok=True)
    with open(a.out, "w") as f:
        json.dump(rows, f)


if __name__ == "__main__":
    main()
