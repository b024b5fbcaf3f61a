"""The allocation-free gradient-statistics entry point.

mdq_grad_stats_multi_noalloc serves callers that cannot allocate device
memory themselves (a host program binding the C ABI with no device allocator
of its own, or a step that must not call cudaMalloc in the middle of its
work): its scratch is a fixed array inside the library.  This file checks it
through the C ABI against the workspace-taking entry point, on two calls in a
row (the second call must not see the first call's scratch contents), and
checks that oversized calls are refused.  It is named so that pytest collects
it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from mdq_b200 import _lib, kernels

pytestmark = pytest.mark.gpu


def _call_noalloc(grads):
    lib = _lib.load()
    n = len(grads)
    ptrs = (ctypes.c_void_p * n)(*[g.data_ptr() for g in grads])
    counts = (ctypes.c_int64 * n)(*[g.numel() for g in grads])
    out = torch.full((n, 4), float("nan"), dtype=torch.float64, device=grads[0].device)
    dt = _lib.MDQ_BF16 if grads[0].dtype == torch.bfloat16 else _lib.MDQ_F32
    st = lib.mdq_grad_stats_multi_noalloc(ptrs, counts, n, dt, out.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream)
    _lib.check(st)
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_entry_point_twice(cuda_device, dtype):
    gen = torch.Generator().manual_seed(7)
    for call in range(2):
        sizes = [(1 << 20) + 11, 3, 70_000, 65_536] if call == 0 else [5, 200_001, 1 << 16]
        grads = [(torch.randn(n, generator=gen) * (1e-3 * (call + 1))).to(dtype).to(cuda_device)
                 for n in sizes]
        got = _call_noalloc(grads)
        want = kernels.grad_stats(grads)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=1e-12)
        # Same records, same fixed summation order: in fact bit-identical.
        assert torch.equal(got.view(torch.int64), want.view(torch.int64)), f"call {call}"


def test_noalloc_refuses_calls_beyond_its_scratch(cuda_device):
    """65537 one-element tensors need 65537 partial records, one more than the
    built-in scratch holds.  Every pointer is a real element of one buffer, so
    even a broken size guard would only read valid memory."""
    lib = _lib.load()
    n = 65537
    g = torch.zeros(n, device=cuda_device)
    ptrs = (ctypes.c_void_p * n)(*[g.data_ptr() + 4 * i for i in range(n)])
    counts = (ctypes.c_int64 * n)(*([1] * n))
    out = torch.full((n, 4), 7.0, dtype=torch.float64, device=cuda_device)
    st = lib.mdq_grad_stats_multi_noalloc(ptrs, counts, n, _lib.MDQ_F32, out.data_ptr(), None)
    torch.cuda.synchronize()
    assert st == _lib.MDQ_ERR_TOO_LARGE
    assert "scratch holds 65536" in lib.mdq_last_error().decode()
    assert bool((out == 7.0).all()), "a refused call must not write its output"
