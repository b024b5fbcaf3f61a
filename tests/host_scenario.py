"""Seeded optimizer scenarios shared by the golden generator and the tests.

Each scenario builds a handful of CPU parameters of awkward sizes, gives each
a gradient of its own scale per step (so the score policy spreads them over
several bit widths and changes its mind on decision steps), runs the
optimizer class and records what the reference's host logic decides.
"""
from __future__ import annotations

import numpy as np
import torch

# Eight tensors of awkward sizes plus 24 small ones with tiny gradients: the
# averages the score compares against are taken over all 32, so the large
# tensors can score high enough for 16 and 32 bits.
SIZES = [127, 1000, 4096 + 17, 300 * 7, 2048, 64 * 65, 3000, 2] + [33] * 24
# Per-parameter gradient scales and densities (a sparse, large gradient has a
# large std / mean|g| ratio and a large RMS, hence a high score).
SCALES = [1e-3, 3e-3, 1e-4, 5e-3, 2e-2, 2e-5, 0.3, 1e-3] + [1e-6] * 24
DENSITY = [1.0, 1.0, 1.0, 1.0, 0.3, 1.0, 0.02, 1.0] + [1.0] * 24

SCENARIOS = {
    "fusedio_b256": dict(cls="fusedio", block_size=256, steps=25, update_freq=20, wd=0.01),
    "simple_b256": dict(cls="simple", block_size=256, steps=25, update_freq=20, wd=0.01),
    "fusedio_b100_uf5": dict(cls="fusedio", block_size=100, steps=24, update_freq=5, wd=0.0),
    "fusedio_b2048": dict(cls="fusedio", block_size=2048, steps=22, update_freq=10, wd=0.1),
    # A one-element tensor has std = NaN: its score, and through the shared
    # EMAs every score, turns NaN and every tensor falls to 4 bits.
    "fusedio_nan": dict(cls="fusedio", block_size=256, steps=6, update_freq=20, wd=0.01,
                        sizes=[1, 500, 64]),
}

DTYPE_CODE = {torch.uint8: 0, torch.int8: 1, torch.int16: 2, torch.uint16: 3, torch.int32: 4,
              torch.uint32: 5}


def make_params(sizes, seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    return [torch.nn.Parameter(torch.randn(n, generator=g) * 0.02) for n in sizes]


def grads_for_step(sizes, step: int, seed: int = 0):
    g = torch.Generator().manual_seed(seed * 1000 + step)
    out = []
    for i, n in enumerate(sizes):
        s, dens = SCALES[i % len(SCALES)], DENSITY[i % len(DENSITY)]
        # vary the relative scales over time so decisions move
        f = s * (1.0 + 0.8 * np.sin(0.7 * step + i))
        x = torch.randn(n, generator=g) * f
        if dens < 1.0:
            x = x * (torch.rand(n, generator=g) < dens).float()
        out.append(x)
    return out


def run_scenario(cls, sc, **extra):
    sizes = sc.get("sizes", SIZES)
    params = make_params(sizes)
    half = (len(params) + 1) // 2
    opt = cls([{"params": params[:half]},
               {"params": params[half:], "weight_decay": 0.0}],
              lr=1e-3, weight_decay=sc["wd"], layer_count=12, batch_size=16,
              update_freq=sc["update_freq"], block_size=sc["block_size"], **extra)
    bits, steps, dtm, dtv, scores = [], [], [], [], []
    for t in range(1, sc["steps"] + 1):
        for p, gr in zip(params, grads_for_step(sizes, t)):
            p.grad = gr.clone()
        opt.step()
        st = [opt.state[p] for p in params]
        bits.append([int(s["current_bit"]) for s in st])
        steps.append([int(s["step"]) for s in st])
        dtm.append([DTYPE_CODE[s["exp_avg"].dtype] for s in st])
        dtv.append([DTYPE_CODE[s["exp_avg_sq"].dtype] for s in st])
        scores.append([float(s["last_score"]) for s in st])
    rec = dict(bits=np.array(bits), steps=np.array(steps), dtype_m=np.array(dtm),
               dtype_v=np.array(dtv), scores=np.array(scores, dtype=np.float32),
               total_steps=np.array(opt.total_steps))
    for i, p in enumerate(params):
        s = opt.state[p]
        rec[f"p{i}"] = p.detach().numpy().copy()
        rec[f"m{i}"] = s["exp_avg"].numpy().view(np.uint8).copy()
        rec[f"v{i}"] = s["exp_avg_sq"].numpy().view(np.uint8).copy()
        for k in ("scale_m", "scale_v", "v_min"):
            rec[f"{k}{i}"] = s[k].numpy().copy()
    return rec
