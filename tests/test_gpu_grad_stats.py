"""Fused gradient statistics (mdq_grad_stats_multi) against float64 sums."""
import numpy as np
import pytest
import torch

from mdq_b200 import kernels

pytestmark = pytest.mark.gpu


def _ref_sums(g: torch.Tensor) -> np.ndarray:
    x = g.float().cpu().numpy().astype(np.float64)
    return np.array([x.sum(), (x * x).sum(), np.abs(x).sum(), x.size])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sums_match_float64(cuda_device, dtype):
    gen = torch.Generator().manual_seed(0)
    sizes = [1, 7, 1000, 65536, 65537, (1 << 20) + 3, 3 * (1 << 16) - 1]
    grads = [(torch.randn(n, generator=gen) * 1e-3 + 2e-4).to(dtype).to(cuda_device)
             for n in sizes]
    out = kernels.grad_stats(grads).cpu().numpy()
    for i, g in enumerate(grads):
        ref = _ref_sums(g)
        np.testing.assert_allclose(out[i, :3], ref[:3], rtol=1e-5, atol=1e-12, err_msg=str(i))
        assert out[i, 3] == ref[3]


def test_deterministic_and_many_tensors(cuda_device):
    gen = torch.Generator().manual_seed(1)
    grads = [torch.randn(((i * 7919) % 5000) + 1, generator=gen).to(cuda_device)
             for i in range(600)]
    a = kernels.grad_stats(grads)
    b = kernels.grad_stats(grads)
    assert torch.equal(a.view(torch.int64), b.view(torch.int64))
    for i in (0, 255, 256, 599):
        np.testing.assert_allclose(a[i, :3].cpu().numpy(), _ref_sums(grads[i])[:3], rtol=1e-5)


def test_unaligned_views(cuda_device):
    base = torch.randn(100_003, device=cuda_device)
    grads = [base[1:70_001], base[3:], base[5:9]]
    out = kernels.grad_stats(grads).cpu().numpy()
    for i, g in enumerate(grads):
        np.testing.assert_allclose(out[i, :3], _ref_sums(g)[:3], rtol=1e-5)
