"""Python face of the CPU oracle (``mdq_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` as the checker; the product never imports
anything under ``oracle/``.

``step`` restates one launch of the reference kernel family
(ruby320/STREAM-MM2026 CUDA/stquant_kernel.cu:53-401) on host arrays.
``fused_mdq_adamw_cpu`` has the reference binding's argument list
(CUDA/stquant_core.cpp:3-7) over CPU torch tensors, so the reference's own
optimizer classes can be driven by it on a machine without a GPU.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libmdq_oracle.so")

LAYOUT_PACKED4, LAYOUT_S8U8, LAYOUT_S16U16, LAYOUT_S32U32, LAYOUT_M8V4 = range(5)

_lib = None


def build(force: bool = False) -> str:
    """Compile libmdq_oracle.so with oracle/Makefile (gcc, no GPU needed)."""
    src = os.path.join(HERE, "mdq_oracle.c")
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "libmdq_oracle.so"], check=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(LIB)
        vp, f, i32, i64 = ctypes.c_void_p, ctypes.c_float, ctypes.c_int, ctypes.c_int64
        lib.mdq_oracle_step.restype = i32
        lib.mdq_oracle_step.argtypes = [vp, vp, i32, vp, vp, vp, vp, vp, i64, i32,
                                        f, f, f, f, f, i32, i32, i32, i32]
        lib.mdq_oracle_grad_sums.restype = None
        lib.mdq_oracle_grad_sums.argtypes = [vp, i64, vp]
        lib.mdq_oracle_max_threads.restype = i32
        lib.mdq_oracle_max_threads.argtypes = []
        _lib = lib
    return _lib


def max_threads() -> int:
    return load().mdq_oracle_max_threads()


def _p(a: np.ndarray | None):
    if a is None or a.size == 0:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def step(p: np.ndarray, grad: np.ndarray, layout: int, m_codes: np.ndarray,
         v_codes: np.ndarray | None, scale_m: np.ndarray, scale_v: np.ndarray,
         v_min: np.ndarray, block: int, beta1: float, beta2: float, lr: float,
         weight_decay: float, eps: float, step: int, m_bits: int, v_bits: int,
         threads: int = 1) -> None:
    """In-place oracle step on numpy arrays; grad float32 (bf16 widened by caller)."""
    assert p.dtype == np.float32 and grad.dtype == np.float32
    for a in (scale_m, scale_v, v_min):
        assert a.dtype == np.float32
    rc = load().mdq_oracle_step(_p(p), _p(grad), layout, _p(m_codes), _p(v_codes),
                                _p(scale_m), _p(scale_v), _p(v_min), p.size, block,
                                beta1, beta2, lr, weight_decay, eps, step, m_bits, v_bits,
                                threads)
    if rc != 0:
        raise ValueError("oracle step rejected its arguments")


def grad_sums(g: np.ndarray) -> np.ndarray:
    """sum g, sum g^2, sum |g|, count (float64)."""
    out = np.zeros(4, np.float64)
    g = np.ascontiguousarray(g, dtype=np.float32)
    load().mdq_oracle_grad_sums(_p(g), g.size, _p(out))
    return out


def fused_mdq_adamw_cpu(p, grad, exp_avg, exp_avg_sq, scale_m, scale_v, v_min,
                        beta1, beta2, lr, weight_decay, eps, step_, bits, block_size,
                        profile_cycles=None):
    """Reference binding's argument list over CPU torch tensors (in place).

    Dispatch as CUDA/stquant_kernel.cu:430-463; block = min(block_size, 1024)
    as :421.  profile_cycles is accepted and left untouched.
    """
    import torch

    T = min(int(block_size), 1024)
    if bits == 4 and exp_avg.dtype == torch.uint8 and exp_avg_sq.numel() == 0:
        layout = LAYOUT_PACKED4
    elif exp_avg.dtype == torch.int8 and exp_avg_sq.dtype == torch.uint8:
        layout = LAYOUT_S8U8
    elif exp_avg.dtype == torch.int16 and exp_avg_sq.dtype == torch.uint16:
        layout = LAYOUT_S16U16
    elif exp_avg.dtype == torch.int32 and exp_avg_sq.dtype == torch.uint32:
        layout = LAYOUT_S32U32
    else:
        raise RuntimeError(f"MDQ: unsupported state {exp_avg.dtype}/{exp_avg_sq.dtype} bits={bits}")
    for t in (p, grad, exp_avg, exp_avg_sq, scale_m, scale_v, v_min):
        assert t.device.type == "cpu" and (t.numel() == 0 or t.is_contiguous())
    g = grad.detach().float().contiguous()
    vp = lambda t: t.data_ptr() if t.numel() else None  # noqa: E731
    rc = load().mdq_oracle_step(vp(p), vp(g), layout, vp(exp_avg), vp(exp_avg_sq),
                                vp(scale_m), vp(scale_v), vp(v_min), p.numel(), T,
                                float(beta1), float(beta2), float(lr), float(weight_decay),
                                float(eps), int(step_), int(bits), int(bits), 1)
    if rc != 0:
        raise RuntimeError("oracle step rejected its arguments")
