"""The fused step's codes and scales are exact only if two facts about CUDA's
logf hold for every input it can see: logf is monotone (block extremes of
logf are logf of extremes) and the lg2.approx-based approximation stays within
its stated bound.  Check both exhaustively on the GPU: every float from 1e-12
to +inf, about 1.4e9 values."""
import ctypes
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def test_logf_monotone_and_filter_bound_hold_for_every_float(tmp_path, cuda_device):
    so = tmp_path / "log_filter_check.so"
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "-Xcompiler", "-fPIC", "-shared",
                    f"-I{os.path.join(REPO, 'include')}",
                    f"-I{os.path.join(REPO, 'stream-mm2026_b200', 'csrc')}",
                    "-o", str(so), os.path.join(HERE, "gpu_support", "log_filter_check.cu")],
                   check=True)
    lib = ctypes.CDLL(str(so))
    out = (ctypes.c_double * 3)()
    assert lib.mdq_check_log_filter(out) == 0
    violations, worst, nonmono = out[0], out[1], out[2]
    print(f"log filter: {violations:.0f} bound violations, worst |a - logf| / tol = {worst:.4f}, "
          f"{nonmono:.0f} monotonicity violations")
    assert nonmono == 0
    assert violations == 0
    assert worst < 1.0
