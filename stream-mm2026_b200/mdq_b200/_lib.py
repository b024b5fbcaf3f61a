"""ctypes binding of the C ABI in ``include/mdq.h`` (``libmdq.so``).

Loading fails loudly when the library is missing: there is no CPU or PyTorch
fallback for the step.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmdq.so")

# mdq_status
MDQ_OK = 0
MDQ_ERR_INVALID_ARG = 1
MDQ_ERR_UNSUPPORTED = 2
MDQ_ERR_CUDA = 3
MDQ_ERR_TOO_LARGE = 4

# mdq_dtype
MDQ_F32, MDQ_BF16, MDQ_I8, MDQ_U8, MDQ_I16, MDQ_U16, MDQ_I32, MDQ_U32 = range(8)

# mdq_layout
LAYOUT_PACKED4, LAYOUT_S8U8, LAYOUT_S16U16, LAYOUT_S32U32, LAYOUT_M8V4 = range(5)

# mdq_p_mode
P_FAST, P_EXACT = 0, 1

ABI_VERSION = 3


class TensorDesc(ctypes.Structure):
    """Mirror of ``mdq_tensor_desc``."""

    _fields_ = [
        ("p", ctypes.c_void_p),
        ("grad", ctypes.c_void_p),
        ("exp_avg", ctypes.c_void_p),
        ("exp_avg_sq", ctypes.c_void_p),
        ("scale_m", ctypes.c_void_p),
        ("scale_v", ctypes.c_void_p),
        ("v_min", ctypes.c_void_p),
        ("n", ctypes.c_int64),
        ("step", ctypes.c_int32),
        ("block", ctypes.c_int32),
        ("lr", ctypes.c_float),
        ("weight_decay", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("beta1", ctypes.c_float),
        ("beta2", ctypes.c_float),
        ("m_bits", ctypes.c_int32),
        ("v_bits", ctypes.c_int32),
        ("layout", ctypes.c_int32),
        ("grad_dtype", ctypes.c_int32),
        ("p_bf16", ctypes.c_void_p),
    ]


class FQDesc(ctypes.Structure):
    """Mirror of ``mdq_fq_desc``."""

    _fields_ = [
        ("p", ctypes.c_void_p),
        ("grad", ctypes.c_void_p),
        ("exp_avg", ctypes.c_void_p),
        ("exp_avg_sq", ctypes.c_void_p),
        ("n", ctypes.c_int64),
        ("block", ctypes.c_int32),
        ("bits", ctypes.c_int32),
        ("grad_dtype", ctypes.c_int32),
        ("apply_decay", ctypes.c_int32),
        ("beta1", ctypes.c_float),
        ("one_minus_beta1", ctypes.c_float),
        ("beta2", ctypes.c_float),
        ("one_minus_beta2", ctypes.c_float),
        ("decay", ctypes.c_float),
        ("step_size", ctypes.c_float),
        ("inv_sqrt_bc2", ctypes.c_float),
        ("eps", ctypes.c_float),
    ]


class StepOptions(ctypes.Structure):
    """Mirror of ``mdq_step_options``."""

    _fields_ = [("p_mode", ctypes.c_int32), ("profile_cycles", ctypes.c_void_p),
                ("n_peers", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("peer_delta", ctypes.c_int64 * 7),
                ("n_grad_ranks", ctypes.c_int32), ("grad_scale", ctypes.c_float),
                ("grad_delta", ctypes.c_int64 * 8)]


class MDQError(RuntimeError):
    """A non-zero mdq_status, with the library's message."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"mdq status {status}: {msg}")
        self.status = status


# Every exported symbol and its signature; tests check the .so exports them all.
_SIGNATURES = {
    "mdq_adamw_step_multi": (ctypes.c_int,
                             [ctypes.POINTER(TensorDesc), ctypes.c_int32,
                              ctypes.POINTER(StepOptions), ctypes.c_void_p]),
    "mdq_fused_adamw": (ctypes.c_int,
                        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                         ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                         ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                         ctypes.c_int64,
                         ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                         ctypes.c_float,
                         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                         ctypes.c_void_p, ctypes.c_void_p]),
    "mdq_grad_stats_workspace_bytes": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int64), ctypes.c_int32,
                                                       ctypes.POINTER(ctypes.c_int64)]),
    "mdq_grad_stats_multi": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p),
                                            ctypes.POINTER(ctypes.c_int64), ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_int64, ctypes.c_void_p]),
    "mdq_grad_stats_multi_noalloc": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p),
                                                    ctypes.POINTER(ctypes.c_int64), ctypes.c_int32,
                                                    ctypes.c_int32, ctypes.c_void_p,
                                                    ctypes.c_void_p]),
    "mdq_fakequant_adamw_multi": (ctypes.c_int, [ctypes.POINTER(FQDesc), ctypes.c_int32,
                                                 ctypes.c_void_p]),
    "mdq_last_error": (ctypes.c_char_p, []),
    "mdq_abi_version": (ctypes.c_int32, []),
}

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return os.environ.get("MDQ_LIB", LIB_PATH)


def load() -> ctypes.CDLL:
    """Load libmdq.so once; raises if it is absent or of another ABI version."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            raise RuntimeError(
                f"MDQ CUDA library not found at {path}; build it with "
                "`python -m mdq_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        ver = lib.mdq_abi_version()
        if ver != ABI_VERSION:
            raise RuntimeError(f"libmdq ABI {ver} != expected {ABI_VERSION}")
        _lib = lib
    return _lib


def check(status: int) -> None:
    if status != MDQ_OK:
        msg = load().mdq_last_error().decode(errors="replace")
        raise MDQError(status, msg)


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)
