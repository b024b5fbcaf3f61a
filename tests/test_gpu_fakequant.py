"""MDQAdamWFakeQuant against the reference's own pure-PyTorch MDQAdamW
(baseline/mdqbock_newhook.py, unmodified, byte-compiled into oracle/_ref),
both on the GPU from the same seeded state and gradients.

The reference class runs its torch operations on CUDA tensors; ours runs one
fused kernel (mdq_fakequant_adamw_multi).  Required after 20 steps: the same
bit widths chosen at every step, and the fp32 moments and the parameters
bit-identical.
"""
import pytest
import torch

from mdq_b200 import MDQAdamWFakeQuant

pytestmark = pytest.mark.gpu


def _reference_class():
    from oracle import build_ref

    return build_ref.load_python_module("mdqbock_newhook").MDQAdamW


def _run(cls, sizes, block, steps, device, **kw):
    g = torch.Generator().manual_seed(0)
    params = [torch.nn.Parameter((torch.randn(n, generator=g) * 0.02).to(device)) for n in sizes]
    opt = cls([{"params": params[:2]}, {"params": params[2:], "weight_decay": 0.0}], lr=1e-3,
              betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, block_size=block, **kw)
    gen = torch.Generator().manual_seed(1)
    bits = []
    for t in range(steps):
        for i, p in enumerate(params):
            scale = 1e-3 * (1 + 4 * (i % 3)) * (1.0 + 0.5 * (t % 4))
            p.grad = (torch.randn(p.numel(), generator=gen) * scale).to(device)
        opt.step()
        bits.append([int(opt.state[p]["current_bit"]) for p in params])
    return params, opt, bits


@pytest.mark.parametrize("sizes,block", [([2048 * 2048], 2048),
                                         ([100_003, 4096 + 17, 777, 2048, 65_536 * 3 + 5], 2048),
                                         ([100_003, 4096 + 17, 777, 3], 100),
                                         ([50_000, 12_345, 999], 4096)])
def test_fakequant_matches_reference_class(cuda_device, sizes, block):
    ref_cls = _reference_class()
    pr, orf, br = _run(ref_cls, sizes, block, 20, cuda_device)
    pm, om, bm = _run(MDQAdamWFakeQuant, sizes, block, 20, cuda_device, grad_stats="reference")
    diff = {k: sum(int((orf.state[a][k].view(torch.int32) != om.state[b][k].view(torch.int32))
                       .sum()) for a, b in zip(pr, pm)) for k in ("exp_avg", "exp_avg_sq")}
    diff["p"] = sum(int((a.detach().view(torch.int32) != b.detach().view(torch.int32)).sum())
                    for a, b in zip(pr, pm))
    print(f"sizes {sizes} block {block}: elements differing {diff}")
    assert bm == br
    same = 0
    for a, b in zip(pr, pm):
        sa, sb = orf.state[a], om.state[b]
        assert sa["step"] == sb["step"]
        for k in ("exp_avg", "exp_avg_sq"):
            assert torch.equal(sa[k].view(torch.int32), sb[k].view(torch.int32)), k
        same += int((a.detach().view(torch.int32) == b.detach().view(torch.int32)).sum())
        assert torch.equal(a.detach().view(torch.int32), b.detach().view(torch.int32))
    total = sum(sizes)
    print(f"sizes {sizes} block {block}: bits {sorted({x for r in br for x in r})}, "
          f"parameters bit-identical {same}/{total}")
