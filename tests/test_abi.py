"""The C-ABI library on a machine without a GPU: it loads, exports every entry
point ``include/mdq.h`` declares, and rejects bad arguments with the
documented status codes before touching CUDA."""
import ctypes
import os
import re

import pytest

from mdq_b200 import _lib
from mdq_b200._lib import MDQ_ERR_INVALID_ARG, MDQ_ERR_UNSUPPORTED, StepOptions, TensorDesc

HEADER_DIR = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include")


def header_functions():
    names = []
    for h in sorted(os.listdir(HEADER_DIR)):
        text = open(os.path.join(HEADER_DIR, h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(mdq_[a-z_0-9]+)\s*\(", text,
                            flags=re.M)
    return names


def test_header_declares_entry_points():
    names = header_functions()
    assert "mdq_adamw_step_multi" in names and "mdq_fused_adamw" in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in header_functions():
        assert hasattr(lib, name), name
    assert set(header_functions()) <= set(_lib.exported_symbols())
    assert lib.mdq_abi_version() == _lib.ABI_VERSION


def _desc(**kw):
    d = TensorDesc()
    d.p = d.grad = d.exp_avg = d.exp_avg_sq = d.scale_m = d.scale_v = d.v_min = 0x1000
    d.n = 100
    d.step = 1
    d.block = 256
    d.lr, d.weight_decay, d.eps, d.beta1, d.beta2 = 1e-3, 0.01, 1e-8, 0.9, 0.999
    d.m_bits = d.v_bits = 8
    d.layout = _lib.LAYOUT_S8U8
    d.grad_dtype = _lib.MDQ_F32
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,status,msg", [
    (dict(n=-1), MDQ_ERR_INVALID_ARG, "negative n"),
    (dict(layout=9), MDQ_ERR_INVALID_ARG, "bad layout"),
    (dict(grad_dtype=_lib.MDQ_I8), MDQ_ERR_UNSUPPORTED, "grad dtype"),
    (dict(p=None), MDQ_ERR_INVALID_ARG, "null pointer"),
    (dict(block=0), MDQ_ERR_UNSUPPORTED, "block"),
    (dict(block=4096), MDQ_ERR_UNSUPPORTED, "block"),
    (dict(block=1500), MDQ_ERR_UNSUPPORTED, "power of two"),
    (dict(m_bits=9), MDQ_ERR_UNSUPPORTED, "m_bits"),
    (dict(layout=_lib.LAYOUT_PACKED4, m_bits=4, v_bits=8), MDQ_ERR_UNSUPPORTED, "v_bits"),
    (dict(layout=_lib.LAYOUT_M8V4, v_bits=4, block=99), MDQ_ERR_UNSUPPORTED, "even block"),
    (dict(step=-3), MDQ_ERR_INVALID_ARG, "negative step"),
])
def test_multi_rejects_bad_descriptors(kw, status, msg):
    lib = _lib.load()
    arr = (TensorDesc * 1)(_desc(**kw))
    st = lib.mdq_adamw_step_multi(arr, 1, None, None)
    assert st == status
    assert msg in lib.mdq_last_error().decode()


def test_multi_rejects_bad_options():
    lib = _lib.load()
    arr = (TensorDesc * 1)(_desc())
    opts = StepOptions(7, None)
    assert lib.mdq_adamw_step_multi(arr, 1, ctypes.byref(opts), None) == MDQ_ERR_INVALID_ARG
    assert lib.mdq_adamw_step_multi(None, 2, None, None) == MDQ_ERR_INVALID_ARG
    # Peer copies: at most 7 peers, deltas non-zero multiples of 16 bytes,
    # and no peers for block sizes that need the per-element kernel.  All are
    # refused before anything touches a device.
    for n_peers, delta, msg in ((8, 16, "n_peers"), (1, 0, "peer_delta"), (1, 24, "peer_delta")):
        opts = StepOptions(0, None)
        opts.n_peers = n_peers
        opts.peer_delta[0] = delta
        assert lib.mdq_adamw_step_multi(arr, 1, ctypes.byref(opts), None) == MDQ_ERR_INVALID_ARG
        assert msg in lib.mdq_last_error().decode()
    for n, delta, msg in ((9, 0, "n_grad_ranks"), (2, 8, "grad_delta")):
        opts = StepOptions(0, None)
        opts.n_grad_ranks, opts.grad_scale = n, 0.5
        opts.grad_delta[1] = delta
        assert lib.mdq_adamw_step_multi(arr, 1, ctypes.byref(opts), None) == MDQ_ERR_INVALID_ARG
        assert msg in lib.mdq_last_error().decode()
    opts = StepOptions(0, None)
    opts.n_peers, opts.peer_delta[0] = 1, 1 << 30
    odd = (TensorDesc * 1)(_desc(block=100))
    assert lib.mdq_adamw_step_multi(odd, 1, ctypes.byref(opts), None) == MDQ_ERR_UNSUPPORTED
    assert "no peer copies" in lib.mdq_last_error().decode()


def test_step_options_layout():
    import ctypes

    assert ctypes.sizeof(StepOptions) == 152
    assert StepOptions.n_peers.offset == 16 and StepOptions.peer_delta.offset == 24
    assert StepOptions.n_grad_ranks.offset == 80 and StepOptions.grad_delta.offset == 88


def test_empty_step_is_a_no_op():
    lib = _lib.load()
    assert lib.mdq_adamw_step_multi(None, 0, None, None) == 0
    arr = (TensorDesc * 1)(_desc(n=0))
    assert lib.mdq_adamw_step_multi(arr, 1, None, None) == 0


def test_reference_signature_dispatch_errors():
    """mdq_fused_adamw mirrors the reference dispatch's TORCH_CHECK
    (CUDA/stquant_kernel.cu:460-463) and packed4 numel check (:432)."""
    lib = _lib.load()
    ptr = 0x1000
    args = lambda ea, eas, ea_n, eas_n, bits: (  # noqa: E731
        ptr, ptr, _lib.MDQ_F32, ptr, ea, ea_n, ptr, eas, eas_n, ptr, ptr, ptr, 100,
        0.9, 0.999, 1e-3, 0.01, 1e-8, 1, bits, 256, None, None)
    st = lib.mdq_fused_adamw(*args(_lib.MDQ_I16, _lib.MDQ_U8, 100, 100, 8))
    assert st == MDQ_ERR_UNSUPPORTED
    assert "state must be packed4" in lib.mdq_last_error().decode()
    st = lib.mdq_fused_adamw(*args(_lib.MDQ_U8, _lib.MDQ_U8, 99, 0, 4))
    assert st == MDQ_ERR_INVALID_ARG
    assert "numel must match" in lib.mdq_last_error().decode()
    st = lib.mdq_fused_adamw(*args(_lib.MDQ_I8, _lib.MDQ_U8, 100, 100, 8)[:20] + (0, None, None))
    assert st == MDQ_ERR_INVALID_ARG


def test_product_has_no_cpu_path():
    """The torch front end refuses CPU tensors instead of computing on them."""
    import torch

    from mdq_b200 import kernels

    p = torch.zeros(10)
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.fused_mdq_adamw(p, p, torch.zeros(10, dtype=torch.int8),
                                torch.zeros(10, dtype=torch.uint8), torch.zeros(1),
                                torch.zeros(1), torch.zeros(1), 0.9, 0.999, 1e-3, 0.0, 1e-8,
                                1, 8, 256)


def test_descriptor_packing_matches_the_ctypes_mirror():
    """fill_desc packs mdq_tensor_desc with struct.pack_into: every field must
    land where the ctypes mirror (and so the C header) has it."""
    import ctypes

    import torch

    from mdq_b200 import kernels
    from mdq_b200._lib import TensorDesc

    assert kernels._DESC_FMT.size == ctypes.sizeof(TensorDesc) == 120
    expect_off = {"p": 0, "grad": 8, "exp_avg": 16, "exp_avg_sq": 24, "scale_m": 32, "scale_v": 40,
                  "v_min": 48, "n": 56, "step": 64, "block": 68, "lr": 72, "weight_decay": 76,
                  "eps": 80, "beta1": 84, "beta2": 88, "m_bits": 92, "v_bits": 96, "layout": 100,
                  "grad_dtype": 104, "p_bf16": 112}
    for name, off in expect_off.items():
        assert getattr(TensorDesc, name).offset == off, name
    p = torch.zeros(1000)
    t = [torch.zeros(1000, dtype=torch.uint8), torch.zeros(4), torch.zeros(4), torch.zeros(4)]
    p16 = torch.zeros(1000, dtype=torch.bfloat16)
    for easq, copy in ((None, None), (torch.zeros(1000, dtype=torch.uint8), p16)):
        it = kernels.StepItem(p=p, grad=torch.zeros(1000, dtype=torch.bfloat16), exp_avg=t[0],
                              exp_avg_sq=easq, scale_m=t[1], scale_v=t[2], v_min=t[3], step=7,
                              block=256, lr=3e-4, weight_decay=0.1, eps=1e-8, beta1=0.9,
                              beta2=0.95, m_bits=8, v_bits=4, layout=4, p_bf16=copy)
        d = TensorDesc()
        kernels.fill_desc(d, it)
        assert (d.p, d.grad, d.exp_avg, d.scale_m, d.scale_v, d.v_min) == (
            p.data_ptr(), it.grad.data_ptr(), t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(),
            t[3].data_ptr())
        assert (d.exp_avg_sq or 0) == (easq.data_ptr() if easq is not None else 0)
        assert (d.n, d.step, d.block, d.m_bits, d.v_bits, d.layout) == (1000, 7, 256, 8, 4, 4)
        assert d.grad_dtype == kernels._DTYPE_CODE[torch.bfloat16]
        assert (d.p_bf16 or 0) == (copy.data_ptr() if copy is not None else 0)
        for name, val in (("lr", 3e-4), ("weight_decay", 0.1), ("eps", 1e-8), ("beta1", 0.9),
                          ("beta2", 0.95)):
            assert getattr(d, name) == ctypes.c_float(val).value, name
