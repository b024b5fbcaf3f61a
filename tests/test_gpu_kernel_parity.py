"""Kernel parity on the GPU: the sm_100a step against the reference's own kernel.

The reference kernel (CUDA/stquant_kernel.cu, built from its sources into
oracle/_ref) and ours start from the same state and see the same gradients
for several steps.  Codes and block scales must be bit-identical at every
step; parameters bit-identical in exact mode and within 1e-6 of max|p| after
20 steps in fast mode (the parameter tolerance the task states).
"""
import pytest
import torch

from mdq_testlib import State, grads, load_reference_kernel
from mdq_b200 import kernels
from mdq_b200.kernels import (LAYOUT_M8V4, LAYOUT_PACKED4, LAYOUT_S8U8, LAYOUT_S16U16,
                              LAYOUT_S32U32, P_EXACT, P_FAST, StepItem)

pytestmark = pytest.mark.gpu

LAYOUT_ID = {"packed4": LAYOUT_PACKED4, "s8u8": LAYOUT_S8U8, "s16u16": LAYOUT_S16U16,
             "s32u32": LAYOUT_S32U32}
HP = dict(beta1=0.9, beta2=0.999, lr=1e-3, weight_decay=0.01, eps=1e-8)


@pytest.fixture(scope="module")
def ref():
    return load_reference_kernel()


def run_ref(ref, st: State, g, step, bits):
    prof = torch.empty(0, dtype=torch.int64, device=st.p.device)
    ref.fused_mdq_adamw(st.p, g.float(), st.m, st.v, st.sm, st.sv, st.vmin, HP["beta1"],
                        HP["beta2"], HP["lr"], HP["weight_decay"], HP["eps"], step, bits,
                        st.block, prof)


def item_of(st: State, g, step, m_bits, v_bits, layout, block=None):
    return StepItem(p=st.p, grad=g, exp_avg=st.m, exp_avg_sq=st.v if st.v.numel() else None,
                    scale_m=st.sm, scale_v=st.sv, v_min=st.vmin, step=step,
                    block=block or st.block, m_bits=m_bits, v_bits=v_bits, layout=layout, **HP)


CASES = [
    # layout, bits, n, block
    ("packed4", 4, 1 << 20, 256),
    ("packed4", 4, 100_003, 128),
    ("packed4", 4, 4096 + 17, 1024),
    ("packed4", 4, 1, 256),
    ("packed4", 4, 127, 32),
    ("packed4", 4, 5000, 8),
    ("packed4", 4, 70_001, 16),
    ("s8u8", 8, 140_003, 1024),
    ("s8u8", 8, 1 << 20, 256),
    ("s8u8", 8, 70_001, 1024),
    ("s8u8", 8, 70_001, 512),
    ("s8u8", 4, 33_333, 64),
    ("s16u16", 16, 200_000, 256),
    ("s16u16", 8, 20_000, 128),
    ("s32u32", 32, 100_000, 256),
    ("s32u32", 16, 9_999, 1024),
    # block sizes that are not powers of two, or below 8: tree kernel
    ("packed4", 4, 10_007, 100),
    ("s8u8", 8, 10_007, 1000),
    ("s16u16", 16, 1_001, 3),
    ("s8u8", 8, 999, 1),
    ("s32u32", 32, 4_000, 6),
]


@pytest.mark.parametrize("layout,bits,n,block", CASES)
@pytest.mark.parametrize("gdt", [torch.float32, torch.bfloat16])
def test_reference_signature_bit_exact(ref, cuda_device, layout, bits, n, block, gdt):
    """kernels.fused_mdq_adamw (reference argument list) == reference kernel."""
    a = State(n, block, layout, cuda_device, seed=n)
    b = a.clone()
    steps = 6
    for s, g in enumerate(grads(n, steps, cuda_device, gdt, seed=block), start=1):
        run_ref(ref, a, g, s, bits)
        kernels.fused_mdq_adamw(b.p, g, b.m, b.v, b.sm, b.sv, b.vmin, HP["beta1"], HP["beta2"],
                                HP["lr"], HP["weight_decay"], HP["eps"], s, bits, block)
        torch.cuda.synchronize()
        mm = a.mismatches(b)
        assert all(v == 0 for v in mm.values()), f"step {s}: {mm}"


@pytest.mark.parametrize("layout,bits,block", [("packed4", 4, 256), ("s8u8", 8, 1024),
                                                ("s16u16", 16, 128), ("packed4", 4, 1024)])
def test_fast_p_mode_20_steps(ref, cuda_device, layout, bits, block):
    """Fast parameter arithmetic: codes/scales exact, p within 1e-6 after 20 steps."""
    n = 300_001
    a = State(n, block, layout, cuda_device, seed=3)
    b = a.clone()
    for s, g in enumerate(grads(n, 20, cuda_device, torch.bfloat16, seed=4), start=1):
        run_ref(ref, a, g, s, bits)
        kernels.step_multi([item_of(b, g, s, bits, bits, LAYOUT_ID[layout])], p_mode=P_FAST)
        torch.cuda.synchronize()
        mm = a.mismatches(b)
        assert all(mm[k] == 0 for k in ("m", "v", "sm", "sv", "vmin")), f"step {s}: {mm}"
    err = (a.p - b.p).abs().max().item()
    assert err <= 1e-6 * a.p.abs().max().item(), err
    rel_l2 = ((a.p - b.p).norm() / a.p.norm()).item()
    assert rel_l2 <= 1e-6, rel_l2


def test_multi_tensor_matches_single(ref, cuda_device):
    """One multi-tensor call over mixed layouts == reference per tensor."""
    spec = [("packed4", 4, 50_000, 256), ("s8u8", 8, 3_000, 128), ("s16u16", 16, 777, 256),
            ("packed4", 4, 2048, 2048 // 2), ("s32u32", 32, 5_000, 64), ("s8u8", 4, 12_345, 100)]
    refs = [State(n, blk, lay, cuda_device, seed=i) for i, (lay, _, n, blk) in enumerate(spec)]
    mine = [r.clone() for r in refs]
    for s in range(1, 5):
        items = []
        for i, ((lay, bits, n, blk), ra, mi) in enumerate(zip(spec, refs, mine)):
            g = grads(n, 1, cuda_device, seed=100 * s + i)[0]
            run_ref(ref, ra, g, s, bits)
            items.append(item_of(mi, g, s, bits, bits, LAYOUT_ID[lay]))
        kernels.step_multi(items, p_mode=P_EXACT)
        torch.cuda.synchronize()
        for ra, mi in zip(refs, mine):
            mm = ra.mismatches(mi)
            assert all(v == 0 for v in mm.values()), f"step {s}: {mm}"


STAGED_CASES = [("s8u8", 8, b) for b in (128, 256, 512, 1024)] + \
    [("packed4", 4, b) for b in (128, 256)]


@pytest.mark.parametrize("layout,bits,block", STAGED_CASES)
@pytest.mark.parametrize("gdt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("p_mode", [P_EXACT, P_FAST])
def test_staged_codes_many_tensors(ref, cuda_device, layout, bits, block, gdt, p_mode):
    """The bulk-copy staged kernels (int8/uint8 codes at 128..1024-element
    blocks, packed 4-bit codes at 128/256 in fast p mode; at 128 and 256 each
    tensor's last n mod 1024 elements go to the tiled kernel), several tensors
    in one call: tensors that start and end inside a CTA's share of units,
    tails, a tensor of one block, one shorter than a block, and one whose m
    codes start 8 bytes past a 16-byte boundary (no bulk copies for it) ==
    reference.  Codes and scales bit for bit; parameters bit for bit in exact
    mode, within 1e-6 of max|p| in fast mode."""
    sizes = [3 * block, 50 * block + 17, 100, 700 * block, block, 5000, 64 * block + 1]
    refs = [State(n, block, layout, cuda_device, seed=i) for i, n in enumerate(sizes)]
    mine = [r.clone() for r in refs]
    odd = mine[1]
    buf = torch.empty(odd.n + 8, dtype=odd.m.dtype, device=cuda_device)
    odd.m = buf[8:8 + odd.n]
    odd.m.copy_(refs[1].m)
    for s in range(1, 6):
        items = []
        for i, (n, ra, mi) in enumerate(zip(sizes, refs, mine)):
            g = grads(n, 1, cuda_device, gdt, seed=100 * s + i)[0]
            run_ref(ref, ra, g, s, bits)
            items.append(item_of(mi, g, s, bits, bits, LAYOUT_ID[layout]))
        kernels.step_multi(items, p_mode=p_mode)
        torch.cuda.synchronize()
        for i, (ra, mi) in enumerate(zip(refs, mine)):
            mm = ra.mismatches(mi)
            keys = ("p", "m", "v", "sm", "sv", "vmin") if p_mode == P_EXACT else \
                ("m", "v", "sm", "sv", "vmin")
            assert all(mm[k] == 0 for k in keys), f"step {s} tensor {i}: {mm}"
            if p_mode == P_FAST:
                err = (ra.p - mi.p).abs().max().item()
                assert err <= 1e-6 * max(ra.p.abs().max().item(), 1e-30), (i, err)


def test_many_tensors_one_launch(ref, cuda_device):
    """More descriptors than one launch holds (224) still match."""
    sizes = [(i * 37) % 900 + 1 for i in range(300)]
    refs = [State(n, 128, "packed4", cuda_device, seed=i) for i, n in enumerate(sizes)]
    mine = [r.clone() for r in refs]
    gs = [grads(n, 1, cuda_device, seed=i)[0] for i, n in enumerate(sizes)]
    for ra, g in zip(refs, gs):
        run_ref(ref, ra, g, 1, 4)
    kernels.step_multi([item_of(mi, g, 1, 4, 4, LAYOUT_PACKED4) for mi, g in zip(mine, gs)],
                       p_mode=P_EXACT)
    torch.cuda.synchronize()
    for ra, mi in zip(refs, mine):
        mm = ra.mismatches(mi)
        assert all(v == 0 for v in mm.values()), mm


@pytest.mark.parametrize("block", [128, 256, 1024])
def test_mixed_m8_v4_codes(ref, cuda_device, block):
    """8-bit m + 4-bit v: m codes equal an all-8-bit reference run's, v codes an
    all-4-bit run's (m and v never depend on each other in the step)."""
    n = 100_000
    r8 = State(n, block, "s8u8", cuda_device, seed=5)
    r4 = State(n, block, "packed4", cuda_device, seed=5)
    mine_m = torch.zeros(n, dtype=torch.int8, device=cuda_device)
    mine_v = torch.zeros((n + 1) // 2, dtype=torch.uint8, device=cuda_device)
    nb = (n + block - 1) // block
    sm = torch.zeros(nb, device=cuda_device)
    sv = torch.zeros(nb, device=cuda_device)
    vmin = torch.full((nb,), -20.0, device=cuda_device)
    p = r8.p.clone()
    for s, g in enumerate(grads(n, 5, cuda_device, seed=6), start=1):
        run_ref(ref, r8, g, s, 8)
        run_ref(ref, r4, g, s, 4)
        kernels.step_multi([StepItem(p=p, grad=g, exp_avg=mine_m, exp_avg_sq=mine_v, scale_m=sm,
                                     scale_v=sv, v_min=vmin, step=s, block=block, m_bits=8,
                                     v_bits=4, layout=LAYOUT_M8V4, **HP)], p_mode=P_EXACT)
        torch.cuda.synchronize()
        assert torch.equal(mine_m, r8.m), f"step {s}: m codes"
        assert torch.equal(sm.view(torch.int32), r8.sm.view(torch.int32)), f"step {s}: scale_m"
        v4 = (r4.m >> 4).to(torch.uint8)
        pair = torch.stack([mine_v & 15, mine_v >> 4], 1).flatten()[:n]
        assert torch.equal(pair, v4), f"step {s}: v codes"
        assert torch.equal(sv.view(torch.int32), r4.sv.view(torch.int32)), f"step {s}: scale_v"
        assert torch.equal(vmin.view(torch.int32), r4.vmin.view(torch.int32)), f"step {s}: v_min"


def test_profile_cycles(cuda_device):
    """profile_cycles (reference CUDA/stquant_kernel.cu:403-412) is filled."""
    st = State(1 << 16, 256, "s8u8", cuda_device)
    prof = torch.zeros(5, dtype=torch.int64, device=cuda_device)
    g = grads(st.n, 1, cuda_device)[0]
    kernels.fused_mdq_adamw(st.p, g, st.m, st.v, st.sm, st.sv, st.vmin, 0.9, 0.999, 1e-3,
                            0.01, 1e-8, 1, 8, 256, prof)
    torch.cuda.synchronize()
    assert (prof > 0).all(), prof


def test_errors_raise(cuda_device):
    """Reference TORCH_CHECK conditions raise RuntimeError."""
    st = State(1000, 256, "s8u8", cuda_device)
    g = grads(st.n, 1, cuda_device)[0]
    with pytest.raises(RuntimeError):
        kernels.fused_mdq_adamw(st.p, g, st.m.to(torch.int16), st.v, st.sm, st.sv, st.vmin, 0.9,
                                0.999, 1e-3, 0.01, 1e-8, 1, 8, 256)
    with pytest.raises(RuntimeError):
        kernels.fused_mdq_adamw(st.p.cpu(), g, st.m, st.v, st.sm, st.sv, st.vmin, 0.9, 0.999,
                                1e-3, 0.01, 1e-8, 1, 8, 256)
    with pytest.raises(RuntimeError):
        prof = torch.zeros(3, dtype=torch.int64, device=cuda_device)
        kernels.fused_mdq_adamw(st.p, g, st.m, st.v, st.sm, st.sv, st.vmin, 0.9, 0.999, 1e-3,
                                0.01, 1e-8, 1, 8, 256, prof)


ADVERSARIAL = ["constant", "zero", "nonfinite", "huge", "tiny", "ramp"]


def adversarial_grad(kind, n, step, device):
    g = torch.Generator().manual_seed(1000 + step)
    if kind == "constant":      # every element of a block equal: all are extremes
        x = torch.full((n,), 1e-3 * (1 + step % 3))
    elif kind == "zero":
        x = torch.zeros(n)
    elif kind == "nonfinite":   # NaN / Inf reach codes, scales and p
        x = torch.randn(n, generator=g) * 1e-3
        x[::997] = float("nan")
        x[5::1499] = float("inf")
        x[7::1777] = -float("inf")
    elif kind == "huge":
        x = torch.randn(n, generator=g) * 1e3
    elif kind == "tiny":
        x = torch.randn(n, generator=g) * 1e-9
    else:                       # smooth ramp: many near-equal neighbours
        x = torch.linspace(-1e-3, 1e-3, n) * (1 + 0.01 * step)
    return x.to(device)


@pytest.mark.parametrize("kind", ADVERSARIAL)
@pytest.mark.parametrize("layout,bits,block", [("packed4", 4, 128), ("packed4", 4, 1024),
                                                ("s8u8", 8, 1024), ("s8u8", 8, 64),
                                                ("s16u16", 16, 256)])
def test_adversarial_inputs_bit_exact(ref, cuda_device, kind, layout, bits, block):
    """Degenerate and non-finite gradients: still bit-identical to the reference
    (NaN compared by bit pattern)."""
    n = 50_000 + 3
    a = State(n, block, layout, cuda_device, seed=11)
    b = a.clone()
    for s in range(1, 5):
        g = adversarial_grad(kind, n, s, cuda_device)
        run_ref(ref, a, g, s, bits)
        kernels.fused_mdq_adamw(b.p, g, b.m, b.v, b.sm, b.sv, b.vmin, HP["beta1"], HP["beta2"],
                                HP["lr"], HP["weight_decay"], HP["eps"], s, bits, block)
        torch.cuda.synchronize()
        mm = a.mismatches(b)
        assert all(v == 0 for v in mm.values()), f"{kind} step {s}: {mm}"


@pytest.mark.parametrize("layout,bits,block", [("packed4", 4, 128), ("s8u8", 8, 1024),
                                                ("s8u8", 8, 256), ("packed4", 4, 2048 // 2)])
def test_long_trajectory_bit_exact(ref, cuda_device, layout, bits, block):
    """40 steps on 1M elements with bf16 gradients of drifting scale."""
    n = (1 << 20) + 77
    a = State(n, block, layout, cuda_device, seed=21)
    b = a.clone()
    gen = torch.Generator().manual_seed(5)
    for s in range(1, 41):
        g = (torch.randn(n, generator=gen) * 1e-3 * (1 + 0.5 * (s % 7))).bfloat16().to(cuda_device)
        run_ref(ref, a, g, s, bits)
        kernels.fused_mdq_adamw(b.p, g, b.m, b.v, b.sm, b.sv, b.vmin, HP["beta1"], HP["beta2"],
                                HP["lr"], HP["weight_decay"], HP["eps"], s, bits, block)
    torch.cuda.synchronize()
    mm = a.mismatches(b)
    assert all(v == 0 for v in mm.values()), mm


@pytest.mark.parametrize("layout,bits,n,block", [("packed4", 4, (1 << 20) + 77, 256),
                                                  ("s8u8", 8, 100_003, 1024),
                                                  ("s16u16", 16, 5_000, 100)])
def test_bf16_parameter_copy(cuda_device, layout, bits, n, block):
    """p_bf16 receives the updated parameters rounded to bf16; everything else
    is what the same step without the copy produces."""
    a = State(n, block, layout, cuda_device, seed=11)
    b = a.clone()
    p16 = torch.full((n,), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    for s, g in enumerate(grads(n, 3, cuda_device, torch.bfloat16, seed=12), start=1):
        kernels.step_multi([item_of(a, g, s, bits, bits, LAYOUT_ID[layout])], p_mode=P_FAST)
        it = item_of(b, g, s, bits, bits, LAYOUT_ID[layout])
        it.p_bf16 = p16
        kernels.step_multi([it], p_mode=P_FAST)
        torch.cuda.synchronize()
        assert all(v == 0 for v in a.mismatches(b).values())
        assert torch.equal(p16.view(torch.int16), b.p.to(torch.bfloat16).view(torch.int16))
