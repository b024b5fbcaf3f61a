"""Optimizer API features beyond the step: robust_quantize against the
reference's pure-PyTorch implementation, checkpoint round trips, getters."""
import io
import os

import numpy as np
import pytest
import torch

from host_scenario import SCENARIOS, grads_for_step, make_params
from mdq_b200 import optim
from test_host_parity import oracle_launch

GOLD = os.path.join(os.path.dirname(__file__), "golden", "robust_quantize.npz")


def test_robust_quantize_matches_reference():
    """MDQAdamW.robust_quantize == baseline/mdqbock_newhook.py:58-83 on the
    committed vectors (bits 4/8/16/32, blocks 2048/256/100, ragged sizes)."""
    g = np.load(GOLD)
    opt = optim.MDQAdamW.__new__(optim.MDQAdamW)
    keys = sorted({k.split("/")[0] for k in g.files})
    for t in keys:
        m = torch.from_numpy(g[f"{t}/m"])
        v = torch.from_numpy(g[f"{t}/v"])
        for bits in (4, 8, 16, 32):
            for block in (2048, 256, 100):
                np.testing.assert_array_equal(opt.robust_quantize(m, bits, False, block).numpy(),
                                              g[f"{t}/m_b{bits}_k{block}"])
                np.testing.assert_array_equal(opt.robust_quantize(v, bits, True, block).numpy(),
                                              g[f"{t}/v_b{bits}_k{block}"])


@pytest.fixture
def cpu_kernel(monkeypatch):
    monkeypatch.setattr(optim.MDQAdamWSimple, "_launch", oracle_launch)
    # CPU tensors: the policy statistics come from the reference's own torch
    # reductions (the fused statistics pass is a CUDA kernel).
    monkeypatch.setattr(optim.MDQAdamWSimple, "_grad_stats_all",
                        lambda self, pwg: [self._compute_grad_stats(p.grad) for p, _ in pwg])
    torch.set_num_threads(1)


def _run(opt_cls, params, steps, start=1, opt=None):
    sizes = [p.numel() for p in params]
    if opt is None:
        opt = opt_cls([{"params": params[:4]}, {"params": params[4:], "weight_decay": 0.0}],
                      lr=1e-3, layer_count=12, batch_size=16, update_freq=5, block_size=256)
    for t in range(start, start + steps):
        for p, g in zip(params, grads_for_step(sizes, t)):
            p.grad = g.clone()
        opt.step()
    return opt


@pytest.mark.parametrize("cls", [optim.MDQAdamWSimple, optim.MDQAdamWSimpleFusedIO])
def test_checkpoint_round_trip_continues_identically(cpu_kernel, cls):
    sizes = SCENARIOS["fusedio_b256"].get("sizes")
    from host_scenario import SIZES
    sizes = sizes or SIZES
    a = make_params(sizes)
    opt_a = _run(cls, a, 12)
    buf = io.BytesIO()
    torch.save({"params": [p.detach().clone() for p in a], "opt": opt_a.state_dict()}, buf)
    _run(cls, a, 10, start=13, opt=opt_a)

    buf.seek(0)
    ck = torch.load(buf, weights_only=False)
    b = [torch.nn.Parameter(t.clone()) for t in ck["params"]]
    opt_b = cls([{"params": b[:4]}, {"params": b[4:], "weight_decay": 0.0}], lr=1e-3,
                layer_count=12, batch_size=16, update_freq=5, block_size=256)
    opt_b.load_state_dict(ck["opt"])
    assert opt_b.total_steps == 12
    _run(cls, b, 10, start=13, opt=opt_b)
    for pa, pb in zip(a, b):
        assert torch.equal(pa.detach().view(torch.int32), pb.detach().view(torch.int32))
    for pa, pb in zip(a, b):
        sa, sb = opt_a.state[pa], opt_b.state[pb]
        assert sa["step"] == sb["step"] and sa["current_bit"] == sb["current_bit"]
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            assert sa[k].dtype == sb[k].dtype and torch.equal(sa[k], sb[k])


def test_state_dict_layout_and_getters(cpu_kernel):
    from host_scenario import SIZES
    params = make_params(SIZES)
    opt = _run(optim.MDQAdamWSimpleFusedIO, params, 6)
    sd = opt.state_dict()
    assert set(sd["mdq_global_stats"]) == {"n_ema", "r_ema", "v_global_ema", "total_steps"}
    for st in sd["state"].values():
        assert {"step", "exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min", "current_bit",
                "last_score"} <= set(st)
        assert st["exp_avg"].dtype in (torch.uint8, torch.int8, torch.int16, torch.int32)
    dist_t = opt.get_bit_distribution()
    dist_w = opt.get_bit_distribution_param_weighted()
    assert abs(sum(dist_t.values()) - 100) < 1e-9 and abs(sum(dist_w.values()) - 100) < 1e-9
    assert 4 <= opt.get_avg_bit_param_weighted() <= 32
    assert len(opt.get_all_raw_scores()) == len(params)
    t = opt.get_last_step_timings()
    for k in ("mdq_stats_ms", "mdq_bit_decision_ms", "quant_dequant_kernel_ms",
              "mdq_fused_io_fast_path_params", "mdq_update_decision"):
        assert k in t
    m, v = opt.dequantized_moments(params[0])
    assert m.shape == (params[0].numel(),) and torch.isfinite(v).all()


@pytest.mark.parametrize("name,cls", [("simple", optim.MDQAdamWSimple),
                                      ("fusedio", optim.MDQAdamWSimpleFusedIO)])
def test_resume_from_reference_written_checkpoint(cpu_kernel, name, cls):
    """A checkpoint written by the reference's own class (params +
    optimizer.state_dict(), tests/golden/make_checkpoint_golden.py) loads into
    ours; continuing gives the reference's continuation bit for bit."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    from make_checkpoint_golden import KW, MORE, SAVE_AT, groups
    from host_scenario import SIZES

    gdir = os.path.join(os.path.dirname(__file__), "golden")
    ck = torch.load(os.path.join(gdir, f"ref_ckpt_{name}.pt"), weights_only=False)
    ref = np.load(os.path.join(gdir, f"ref_ckpt_{name}_final.npz"))
    params = [torch.nn.Parameter(t.clone()) for t in ck["params"]]
    opt = cls(groups(params), **KW)
    opt.load_state_dict(ck["optimizer"])
    for t in range(SAVE_AT + 1, SAVE_AT + MORE + 1):
        for p, g in zip(params, grads_for_step(SIZES, t)):
            p.grad = g.clone()
        opt.step()
    assert opt.total_steps == int(ref["total_steps"])
    for i, p in enumerate(params):
        st = opt.state[p]
        np.testing.assert_array_equal(p.detach().numpy().view(np.int32), ref[f"p{i}"].view(np.int32))
        assert int(st["current_bit"]) == int(ref[f"bits{i}"]) and int(st["step"]) == int(ref[f"step{i}"])
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            tt = st[k]
            assert str(tt.dtype) == str(ref[f"{k}{i}_dtype"]), (i, k)
            got = tt.view(torch.uint8).numpy() if tt.numel() else np.zeros(0, np.uint8)
            np.testing.assert_array_equal(got, ref[f"{k}{i}"], err_msg=f"param {i} {k}")


def test_quant_error_is_the_training_scripts_metric(cpu_kernel):
    """quant_error() == the reference script's compute_mdq_quant_error
    (baseline/pretrain_gpt.py:88-104, restated here) over the decoded moments."""
    from host_scenario import SIZES
    params = make_params(SIZES)
    opt = _run(optim.MDQAdamWSimpleFusedIO, params, 6)
    num = den = 0.0
    for group in opt.param_groups:
        for p in group["params"]:
            st = opt.state[p]
            bit = st.get("current_bit", 32)
            m, v = opt.dequantized_moments(p)
            qm = opt.robust_quantize(m, bit, is_v=False, block_size=256)
            qv = opt.robust_quantize(v, bit, is_v=True, block_size=256)
            num += (m - qm).pow(2).sum().item() + (v - qv).pow(2).sum().item()
            den += m.pow(2).sum().item() + v.pow(2).sum().item()
    want = (num / (den + 1e-12)) ** 0.5
    got = opt.quant_error()
    assert 0.0 < got < 1.0
    assert abs(got - want) <= 1e-5 * want
