"""Host logic of MDQAdamWFakeQuant on CPU against the reference's own
pure-PyTorch MDQAdamW (baseline/mdqbock_newhook.py, unmodified, byte-compiled
into oracle/_ref by the build).

The fused kernel is replaced by a test double that applies, per step item,
the reference's own per-parameter update expressions (:159-170, with the
reference class's robust_quantize) to the tensors the item names.  What is
under test is everything around the kernel: state initialisation, the score
policy and its bit widths, step counting, the block size (never clamped), and
the host scalars handed to the kernel (betas, lr, weight decay, eps, step).
Everything must match the reference class bit for bit.
"""
import math
import os

import pytest
import torch

from mdq_b200 import kernels, optim

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.skipif(
    not os.path.isfile(os.path.join(REPO, "oracle", "_ref", "mdqbock_newhook.pycode")),
    reason="the reference module is not built into oracle/_ref")


def _reference_class():
    from oracle import build_ref

    return build_ref.load_python_module("mdqbock_newhook").MDQAdamW


def _double(ref_cls):
    quant = ref_cls.robust_quantize

    def fakequant_step(items, stream=None):
        for it in items:
            p, g, m, v = it["p"], it["grad"], it["exp_avg"], it["exp_avg_sq"]
            b1, b2, step = it["beta1"], it["beta2"], it["step"]
            m.mul_(b1).add_(g, alpha=1 - b1)
            v.mul_(b2).addcmul_(g, g, value=1 - b2)
            qm = quant(None, m, it["bits"], False, it["block"])
            qv = quant(None, v, it["bits"], True, it["block"])
            if it["weight_decay"] != 0:
                p.data.mul_(1 - it["lr"] * it["weight_decay"])
            bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
            denom = (qv.sqrt() / math.sqrt(bc2)).add_(it["eps"])
            p.data.addcdiv_(qm, denom, value=-it["lr"] / bc1)
    return fakequant_step


def _run(cls, sizes, block, steps, **kw):
    g = torch.Generator().manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(n, generator=g) * 0.02) for n in sizes]
    opt = cls([{"params": params[:2]}, {"params": params[2:], "weight_decay": 0.0}], lr=1e-3,
              betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, block_size=block, **kw)
    gen = torch.Generator().manual_seed(1)
    bits = []
    for t in range(steps):
        for i, p in enumerate(params):
            scale = 1e-3 * (1 + 4 * (i % 3)) * (1.0 + 0.5 * (t % 4))
            p.grad = torch.randn(p.numel(), generator=gen) * scale
        opt.step()
        bits.append([int(opt.state[p]["current_bit"]) for p in params])
    return params, opt, bits


@pytest.mark.parametrize("sizes,block", [([20_000, 4096 + 17, 777, 2048, 9_001], 2048),
                                         ([5_003, 777, 3], 100)])
def test_fakequant_host_logic_matches_reference_class(monkeypatch, sizes, block):
    torch.set_num_threads(1)
    ref_cls = _reference_class()
    monkeypatch.setattr(kernels, "fakequant_step", _double(ref_cls))
    monkeypatch.setattr(torch.cuda, "Event", lambda **kw: _NoEvent())
    monkeypatch.setattr(torch.cuda, "device", lambda d: _NullCtx())
    pr, orf, br = _run(ref_cls, sizes, block, 22)
    pm, om, bm = _run(optim.MDQAdamWFakeQuant, sizes, block, 22, grad_stats="reference")
    assert br == bm
    assert len({b for row in br for b in row}) >= 2
    assert orf.total_steps == om.total_steps
    for a, b in zip(pr, pm):
        sa, sb = orf.state[a], om.state[b]
        assert sa["step"] == sb["step"]
        assert float(sa["last_score"]) == float(sb["last_score"])
        for k in ("exp_avg", "exp_avg_sq"):
            assert torch.equal(sa[k].view(torch.int32), sb[k].view(torch.int32)), k
        assert torch.equal(a.detach().view(torch.int32), b.detach().view(torch.int32))
    sd = om.state_dict()
    assert set(sd["mdq_global_stats"]) == {"n_ema", "r_ema", "v_global_ema", "total_steps"}


class _NoEvent:
    def record(self, *a):
        pass


class _NullCtx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False
