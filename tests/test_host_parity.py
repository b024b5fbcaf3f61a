"""Host-logic parity: mdq_b200's optimizer classes against the reference's.

tests/golden/host_trajectories.npz holds trajectories of the reference's own
classes (CUDA/stquant_opt_simple.py, CUDA/stquant_opt_fused_io.py) driven by
the CPU oracle as their kernel (tests/golden/make_host_golden.py).  Here the
same scenarios run through mdq_b200's classes with the same oracle standing in
for the CUDA launch (a test double swapped in with monkeypatch; the product
has no CPU path).  Everything the host logic decides must match exactly: bit
widths per step, per-parameter step counters (FusedIO's double increment on a
layout change included), storage dtypes, scores, and final codes, scales and
parameters.
"""
import os

import numpy as np
import pytest
import torch

from host_scenario import SCENARIOS, run_scenario
from mdq_b200 import optim
from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "host_trajectories.npz")


def oracle_launch(self, items, device):
    """Run queued step items through the CPU oracle (test double)."""
    for it in items:
        v = it.exp_avg_sq.numpy() if it.exp_avg_sq is not None else None
        oracle.step(it.p.detach().numpy(), it.grad.float().numpy(), it.layout,
                    it.exp_avg.numpy(), v, it.scale_m.numpy(), it.scale_v.numpy(),
                    it.v_min.numpy(), it.block, it.beta1, it.beta2, it.lr, it.weight_decay,
                    it.eps, it.step, it.m_bits, it.v_bits)
        if getattr(it, "p_bf16", None) is not None:
            it.p_bf16.copy_(it.p.to(torch.bfloat16))


def cpu_fused_stats(self, params_with_grad):
    """Test double of the fused statistics pass for CPU tensors: the same
    float64 (sum g, sum g^2, sum |g|, count) rows, then stats_from_sums."""
    rows = []
    for p, _ in params_with_grad:
        g = p.grad.double().reshape(-1)
        rows.append(torch.stack([g.sum(), (g * g).sum(), g.abs().sum(),
                                 torch.tensor(float(g.numel()), dtype=torch.float64)]))
    return list(optim.stats_from_sums(torch.stack(rows)))


@pytest.fixture
def cpu_kernel(monkeypatch):
    monkeypatch.setattr(optim.MDQAdamWSimple, "_launch", oracle_launch)
    # CPU tensors: the policy statistics come from the reference's own torch
    # reductions (the fused statistics pass is a CUDA kernel).
    monkeypatch.setattr(optim.MDQAdamWSimple, "_grad_stats_all",
                        lambda self, pwg: [self._compute_grad_stats(p.grad) for p, _ in pwg])
    torch.set_num_threads(1)


CLASSES = {"simple": optim.MDQAdamWSimple, "fusedio": optim.MDQAdamWSimpleFusedIO}


@pytest.mark.parametrize("name", sorted(SCENARIOS))
def test_trajectory_matches_reference(cpu_kernel, name):
    gold = np.load(GOLDEN)
    sc = SCENARIOS[name]
    rec = run_scenario(CLASSES[sc["cls"]], sc)
    for key, val in rec.items():
        ref = gold[f"{name}/{key}"]
        if val.dtype.kind == "f":
            np.testing.assert_array_equal(val.view(np.int32) if val.dtype == np.float32 else val,
                                          ref.view(np.int32) if ref.dtype == np.float32 else ref,
                                          err_msg=f"{name}/{key}")
        else:
            np.testing.assert_array_equal(val, ref, err_msg=f"{name}/{key}")


def test_golden_covers_policy_paths():
    """The fixture exercises 4/8/16-bit choices, changes of mind and the
    FusedIO double step count, so the comparison above is not vacuous."""
    gold = np.load(GOLDEN)
    bits = np.concatenate([gold[f"{n}/bits"].ravel() for n in SCENARIOS])
    assert {4, 8, 16} <= set(bits.tolist())
    b = gold["fusedio_b100_uf5/bits"]
    assert (b[1:] != b[:-1]).any()
    steps_f = gold["fusedio_b256/steps"][-1]
    steps_s = gold["simple_b256/steps"][-1]
    assert (steps_f > steps_s).any()
    assert (gold["fusedio_nan/bits"] == 4).all()
