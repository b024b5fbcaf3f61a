"""Speed against the reference's own kernel on the same B200 (reported, and
required to be a clear win): one 2^27-element fused step, 4-bit and 8-bit,
block 1024 as the reference's CUDA path clamps it, fp32 gradients for both."""
import pytest
import torch

from mdq_testlib import State, load_reference_kernel
from mdq_b200 import kernels
from mdq_b200.kernels import LAYOUT_PACKED4, LAYOUT_S8U8, P_EXACT, P_FAST, StepItem

pytestmark = pytest.mark.gpu


def _time(fn, iters=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


@pytest.mark.parametrize("layout,bits", [("packed4", 4), ("s8u8", 8)])
def test_faster_than_reference_kernel(cuda_device, layout, bits):
    ref = load_reference_kernel()
    n, block = 1 << 27, 1024
    st = State(n, block, layout, cuda_device)
    g = torch.randn(n, device=cuda_device) * 1e-3
    prof = torch.empty(0, dtype=torch.int64, device=cuda_device)
    t_ref = _time(lambda: ref.fused_mdq_adamw(st.p, g, st.m, st.v, st.sm, st.sv, st.vmin, 0.9,
                                              0.999, 1e-3, 0.01, 1e-8, 5, bits, block, prof))
    lay = LAYOUT_PACKED4 if layout == "packed4" else LAYOUT_S8U8
    it = StepItem(p=st.p, grad=g, exp_avg=st.m, exp_avg_sq=st.v if st.v.numel() else None,
                  scale_m=st.sm, scale_v=st.sv, v_min=st.vmin, step=5, block=block, lr=1e-3,
                  weight_decay=0.01, eps=1e-8, beta1=0.9, beta2=0.999, m_bits=bits, v_bits=bits,
                  layout=lay)
    t_exact = _time(lambda: kernels.step_multi([it], p_mode=P_EXACT))
    t_fast = _time(lambda: kernels.step_multi([it], p_mode=P_FAST))
    gp = lambda t: n / t / 1e6  # noqa: E731
    print(f"{layout}: reference {t_ref:.3f} ms ({gp(t_ref):.1f} Gparams/s), "
          f"exact {t_exact:.3f} ms ({gp(t_exact):.1f}), fast {t_fast:.3f} ms ({gp(t_fast):.1f}); "
          f"speed-up {t_ref / t_fast:.1f}x / {t_ref / t_exact:.1f}x")
    assert t_exact * 4 < t_ref
