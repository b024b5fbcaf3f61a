"""Drop-in stand-in for the reference's extension module ``stquant_timetest_cpp``.

The reference's optimizer classes (CUDA/stquant_opt_simple.py:13,
CUDA/stquant_opt_fused_io.py:10) import ``stquant_timetest_cpp`` and call its
``fused_mdq_adamw`` (bound at CUDA/stquant_core.cpp:9-15).  With this
directory on ``sys.path`` ahead of the reference's build, those classes run
unchanged on the sm_100a kernel: same argument list, in-place semantics, and
RuntimeError where the reference raises.
"""
from mdq_b200.kernels import fused_mdq_adamw  # noqa: F401

__all__ = ["fused_mdq_adamw"]
