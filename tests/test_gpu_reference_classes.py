"""The reference's own optimizer classes against ours, on the GPU, through a model.

The reference side is CUDA/stquant_opt_simple.py:MDQAdamWSimple and
CUDA/stquant_opt_fused_io.py:MDQAdamWSimpleFusedIO exactly as the reference
ships them (byte-compiled into oracle/_ref by oracle/build_ref.py, not
edited), driving the reference's own kernel (CUDA/stquant_kernel.cu, built
into oracle/_ref).  Our side is mdq_b200's MDQAdamWSimple and
MDQAdamWSimpleFusedIO on the sm_100a kernels, in exact parameter mode.

GPT-2 small (random init, bf16 autocast) trains for 30 steps on a learnable
synthetic stream with deterministic backward kernels.  Required, for each
class pair: every loss, every parameter, every tensor's bit width, step
counter, code tensor and block scale identical.  Our classes run twice: with
the reference's float32 torch statistics for the bit policy
(grad_stats="reference"), and with the fused float64 statistics pass (the
default), whose bit decisions must come out the same here.
"""
import os

import pytest
import torch

os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")

from mdq_testlib import load_reference_classes
from mdq_b200 import optim

pytestmark = pytest.mark.gpu

STEPS, MICRO, SEQ = 30, 8, 256
KW = dict(lr=3e-4, layer_count=12, batch_size=MICRO, block_size=256, update_freq=10)


def _model(device):
    from transformers import GPT2Config, GPT2LMHeadModel

    torch.manual_seed(0)
    cfg = GPT2Config()  # 12 layers, d 768, 12 heads, ctx 1024, vocab 50257, tied
    cfg._attn_implementation = "eager"
    return GPT2LMHeadModel(cfg).to(device)


def _train(device, make_opt):
    model = _model(device)
    opt = make_opt(model.parameters())
    gen = torch.Generator(device=device).manual_seed(1)
    losses, bits = [], []
    pos = torch.arange(SEQ, device=device)
    for _ in range(STEPS):
        start = torch.randint(0, 4096, (MICRO, 1), device=device, generator=gen)
        ids = (start * 31 + pos * 7919) % 4096
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(input_ids=ids, labels=ids).loss
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(float(loss.detach()))
        bits.append([int(opt.state[p]["current_bit"]) for p in model.parameters()])
    return losses, bits, list(model.parameters()), opt


def _same_state(ref_run, our_run):
    l_r, b_r, p_r, o_r = ref_run
    l_o, b_o, p_o, o_o = our_run
    assert l_o == l_r
    assert b_o == b_r
    for i, (a, b) in enumerate(zip(p_r, p_o)):
        assert torch.equal(a.detach().view(torch.int32), b.detach().view(torch.int32)), i
        sa, sb = o_r.state[a], o_o.state[b]
        assert int(sa["step"]) == int(sb["step"]), i
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            ta, tb = sa[k], sb[k]
            assert ta.dtype == tb.dtype and ta.shape == tb.shape, (i, k)
            if ta.numel():
                assert torch.equal(ta.view(torch.uint8), tb.view(torch.uint8)), (i, k)


@pytest.mark.parametrize("which", ["simple", "fusedio"])
def test_reference_class_vs_ours_gpt2(cuda_device, which):
    ref_simple, ref_fused = load_reference_classes()
    ref_cls = ref_simple if which == "simple" else ref_fused
    our_cls = optim.MDQAdamWSimple if which == "simple" else optim.MDQAdamWSimpleFusedIO
    was = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True)
    try:
        ref_run = _train(cuda_device, lambda ps: ref_cls(ps, **KW))
        ours_ref_stats = _train(cuda_device, lambda ps: our_cls(ps, p_mode="exact",
                                                                 grad_stats="reference", **KW))
        _same_state(ref_run, ours_ref_stats)
        del ours_ref_stats
        ours_fused = _train(cuda_device, lambda ps: our_cls(ps, p_mode="exact", **KW))
        _same_state(ref_run, ours_fused)
    finally:
        torch.use_deterministic_algorithms(was)
    bits = ref_run[1]
    seen = {b for row in bits for b in row}
    print(which, "bit widths seen:", sorted(seen), "losses", [round(x, 3) for x in ref_run[0][::6]])
    assert len(seen) >= 2, "the policy should pick more than one width here"
    assert ref_run[0][-1] < ref_run[0][0] - 1.0
