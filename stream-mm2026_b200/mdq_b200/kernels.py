"""Torch-tensor front end of the C ABI.

``fused_mdq_adamw`` keeps the exact argument list of the reference binding
``stquant_timetest_cpp.fused_mdq_adamw`` (CUDA/stquant_core.cpp:3-15,
CUDA/stquant_kernel.cu:414-465): it mutates p, the codes and the scales in
place on the current stream and raises RuntimeError where the reference's
TORCH_CHECKs would.  ``step_multi`` updates many tensors in one call.
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import (LAYOUT_M8V4, LAYOUT_PACKED4, LAYOUT_S8U8, LAYOUT_S16U16, LAYOUT_S32U32,
                   P_EXACT, P_FAST, StepOptions, TensorDesc)

_DTYPE_CODE = {
    torch.float32: _lib.MDQ_F32,
    torch.bfloat16: _lib.MDQ_BF16,
    torch.int8: _lib.MDQ_I8,
    torch.uint8: _lib.MDQ_U8,
    torch.int16: _lib.MDQ_I16,
    torch.uint16: _lib.MDQ_U16,
    torch.int32: _lib.MDQ_I32,
    torch.uint32: _lib.MDQ_U32,
}

LAYOUT_NAMES = {
    LAYOUT_PACKED4: "packed4",
    LAYOUT_S8U8: "s8u8",
    LAYOUT_S16U16: "s16u16",
    LAYOUT_S32U32: "s32u32",
    LAYOUT_M8V4: "m8v4",
}


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    if t is None or t.numel() == 0:
        return None
    return t.data_ptr()


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what} must be CUDA")


def _need_contig(t: torch.Tensor, what: str) -> None:
    if not t.is_contiguous():
        raise RuntimeError(f"{what} must be contiguous")


def fused_mdq_adamw(p, grad, exp_avg, exp_avg_sq, scale_m, scale_v, v_min,
                    beta1, beta2, lr, weight_decay, eps, step, bits, block_size,
                    profile_cycles=None):
    """In-place fused MDQ-AdamW step of one tensor (reference argument list)."""
    _need_cuda(p, "p/grad")
    _need_cuda(grad, "p/grad")
    _need_cuda(exp_avg, "exp_avg")
    if p.dtype != torch.float32:
        raise RuntimeError("p must be float32")
    if grad.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError("grad must be float32 or bfloat16")
    for t, name in ((p, "p"), (grad, "grad"), (exp_avg, "exp_avg"), (exp_avg_sq, "exp_avg_sq"),
                    (scale_m, "scale_m"), (scale_v, "scale_v"), (v_min, "v_min")):
        _need_contig(t, name)
    if grad.numel() != p.numel():
        raise RuntimeError("grad numel must match p")
    prof = None
    if profile_cycles is not None and profile_cycles.numel() > 0:
        if not (profile_cycles.is_cuda and profile_cycles.dtype == torch.int64):
            raise RuntimeError("profile_cycles must be CUDA int64 tensor")
        if profile_cycles.numel() < 5:
            raise RuntimeError("profile_cycles needs >= 5 elements")
        prof = profile_cycles.data_ptr()
    ea_code = _DTYPE_CODE.get(exp_avg.dtype, -1)
    eas_code = _DTYPE_CODE.get(exp_avg_sq.dtype, -1)
    lib = _lib.load()
    with torch.cuda.device(p.device):
        st = lib.mdq_fused_adamw(
            p.data_ptr(), grad.data_ptr(), _DTYPE_CODE[grad.dtype],
            _ptr(exp_avg), ea_code, exp_avg.numel(),
            _ptr(exp_avg_sq), eas_code, exp_avg_sq.numel(),
            scale_m.data_ptr(), scale_v.data_ptr(), v_min.data_ptr(),
            p.numel(),
            float(beta1), float(beta2), float(lr), float(weight_decay), float(eps),
            int(step), int(bits), int(block_size), prof, _stream_handle(p.device))
    _lib.check(st)


@dataclass
class StepItem:
    """One tensor, or one block-aligned piece of a tensor, for ``step_multi``."""

    p: torch.Tensor
    grad: torch.Tensor
    exp_avg: torch.Tensor
    exp_avg_sq: Optional[torch.Tensor]
    scale_m: torch.Tensor
    scale_v: torch.Tensor
    v_min: torch.Tensor
    step: int
    block: int
    lr: float
    weight_decay: float
    eps: float
    beta1: float
    beta2: float
    m_bits: int
    v_bits: int
    layout: int
    p_bf16: Optional[torch.Tensor] = None   # bf16 copy of the updated parameters


# mdq_tensor_desc as packed bytes: 7 pointers, int64 n, int32 step / block,
# 5 floats, 4 int32, 4 bytes of padding, one pointer (tests/test_abi.py
# checks the offsets against the ctypes mirror).  One pack_into per descriptor costs
# far less host time than 19 ctypes attribute stores.
_DESC_FMT = struct.Struct("=7Qq2i5f4i4xQ")


def fill_desc(d: TensorDesc, it: StepItem) -> None:
    easq = it.exp_avg_sq
    _DESC_FMT.pack_into(
        d, 0, it.p.data_ptr(), it.grad.data_ptr(), it.exp_avg.data_ptr(),
        easq.data_ptr() if easq is not None and easq.numel() else 0,
        it.scale_m.data_ptr(), it.scale_v.data_ptr(), it.v_min.data_ptr(),
        it.p.numel(), int(it.step), int(it.block), float(it.lr), float(it.weight_decay),
        float(it.eps), float(it.beta1), float(it.beta2), int(it.m_bits), int(it.v_bits),
        int(it.layout), _DTYPE_CODE.get(it.grad.dtype, -1),
        it.p_bf16.data_ptr() if it.p_bf16 is not None else 0)


def run_descs(descs, count: int, device: torch.device, p_mode: int = P_FAST,
              profile_cycles: Optional[torch.Tensor] = None, stream: Optional[int] = None,
              peer_deltas: Optional[Sequence[int]] = None,
              grad_ranks: Optional[tuple] = None) -> None:
    """Launch a prepared ``TensorDesc`` array (the optimizer keeps one alive).
    ``peer_deltas``: byte offsets from each updated parameter's local copy
    (p_bf16, else p) to its copies on other GPUs.  ``grad_ranks``: (scale,
    byte offsets of every rank's gradient buffer in rank order, 0 for this
    rank): the step sums the ranks' gradients and scales the sum
    (mdq_step_options)."""
    opts = StepOptions(p_mode, profile_cycles.data_ptr() if profile_cycles is not None else None)
    if peer_deltas:
        if len(peer_deltas) > 7:
            raise ValueError("at most 7 peers")
        opts.n_peers = len(peer_deltas)
        for k, dlt in enumerate(peer_deltas):
            opts.peer_delta[k] = int(dlt)
    if grad_ranks:
        scale, deltas = grad_ranks
        if len(deltas) > 8:
            raise ValueError("at most 8 gradient ranks")
        opts.n_grad_ranks = len(deltas)
        opts.grad_scale = float(scale)
        for k, dlt in enumerate(deltas):
            opts.grad_delta[k] = int(dlt)
    lib = _lib.load()
    with torch.cuda.device(device):
        st = lib.mdq_adamw_step_multi(descs, count, ctypes.byref(opts),
                                      stream if stream is not None else _stream_handle(device))
    _lib.check(st)


def step_multi(items: Sequence[StepItem], p_mode: int = P_FAST,
               profile_cycles: Optional[torch.Tensor] = None) -> None:
    """Fused MDQ-AdamW step of many tensors on the current stream."""
    if not items:
        return
    arr = (TensorDesc * len(items))()
    dev = items[0].p.device
    for d, it in zip(arr, items):
        for t in (it.p, it.grad, it.exp_avg, it.scale_m, it.scale_v, it.v_min):
            _need_cuda(t, "step tensors")
            _need_contig(t, "step tensors")
            if t.device != dev:
                raise RuntimeError("all tensors of one step_multi call must share a device")
        if it.p_bf16 is not None:
            _need_cuda(it.p_bf16, "p_bf16")
            _need_contig(it.p_bf16, "p_bf16")
            if it.p_bf16.dtype != torch.bfloat16 or it.p_bf16.numel() != it.p.numel():
                raise RuntimeError("p_bf16 must be a bfloat16 tensor of p's size")
        fill_desc(d, it)
    run_descs(arr, len(items), dev, p_mode, profile_cycles)


def grad_stats(grads: Sequence[torch.Tensor]) -> torch.Tensor:
    """(sum g, sum g^2, sum |g|, count) per gradient, float64 [len(grads), 4],
    from one fused pass on the current stream (deterministic).  The scratch
    workspace is allocated here through torch's caching allocator."""
    if not grads:
        return torch.zeros(0, 4, dtype=torch.float64)
    dev = grads[0].device
    dt = grads[0].dtype
    for g in grads:
        _need_cuda(g, "gradients")
        _need_contig(g, "gradients")
        if g.dtype != dt or g.device != dev:
            raise RuntimeError("gradients of one grad_stats call share dtype and device")
    if dt not in (torch.float32, torch.bfloat16):
        raise RuntimeError("gradients must be float32 or bfloat16")
    n = len(grads)
    ptrs = (ctypes.c_void_p * n)(*[g.data_ptr() for g in grads])
    counts = (ctypes.c_int64 * n)(*[g.numel() for g in grads])
    lib = _lib.load()
    need = ctypes.c_int64(0)
    _lib.check(lib.mdq_grad_stats_workspace_bytes(counts, n, ctypes.byref(need)))
    ws = torch.empty(max(need.value, 8), dtype=torch.uint8, device=dev)
    out = torch.empty(n, 4, dtype=torch.float64, device=dev)
    with torch.cuda.device(dev):
        st = lib.mdq_grad_stats_multi(ptrs, counts, n, _DTYPE_CODE[dt], out.data_ptr(),
                                      ws.data_ptr(), need.value, _stream_handle(dev))
    _lib.check(st)
    return out


def layout_for_bits(m_bits: int, v_bits: int) -> int:
    """Storage layout the optimizer uses for a (m_bits, v_bits) pair."""
    if m_bits == v_bits:
        if m_bits <= 4:
            return LAYOUT_PACKED4
        if m_bits <= 8:
            return LAYOUT_S8U8
        if m_bits <= 16:
            return LAYOUT_S16U16
        return LAYOUT_S32U32
    if m_bits <= 8 and v_bits <= 4:
        return LAYOUT_M8V4
    b = max(m_bits, v_bits)
    return layout_for_bits(b, b)


__all__ = ["fused_mdq_adamw", "StepItem", "step_multi", "run_descs", "fill_desc", "grad_stats",
           "layout_for_bits", "P_FAST", "P_EXACT", "LAYOUT_NAMES"]


def fakequant_step(items, stream: Optional[int] = None) -> None:
    """Fused step of the reference's pure-PyTorch MDQAdamW
    (baseline/mdqbock_newhook.py:86-175) for many tensors, on the current
    stream.  Each item is a dict with p, grad, exp_avg, exp_avg_sq (fp32
    moments, updated in place), block, bits, and the host-side scalars of
    the reference's step (beta1, beta2, lr, weight_decay, eps, step)."""
    import math

    if not items:
        return
    arr = (_lib.FQDesc * len(items))()
    dev = items[0]["p"].device
    for d, it in zip(arr, items):
        p, g, m, v = it["p"], it["grad"], it["exp_avg"], it["exp_avg_sq"]
        for t in (p, g, m, v):
            _need_cuda(t, "fake-quant step tensors")
            _need_contig(t, "fake-quant step tensors")
            if t.numel() != p.numel() or t.device != dev:
                raise RuntimeError("p, grad, exp_avg, exp_avg_sq must match in size and device")
        if p.dtype != torch.float32 or m.dtype != torch.float32 or v.dtype != torch.float32:
            raise RuntimeError("p, exp_avg and exp_avg_sq must be float32")
        b1, b2, lr, wd, step = (it["beta1"], it["beta2"], it["lr"], it["weight_decay"],
                                it["step"])
        bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
        d.p, d.grad, d.exp_avg, d.exp_avg_sq = (p.data_ptr(), g.data_ptr(), m.data_ptr(),
                                                v.data_ptr())
        d.n, d.block, d.bits = p.numel(), int(it["block"]), int(it["bits"])
        d.grad_dtype = _DTYPE_CODE.get(g.dtype, -1)
        d.apply_decay = 1 if wd != 0 else 0
        d.beta1, d.one_minus_beta1 = b1, 1 - b1
        d.beta2, d.one_minus_beta2 = b2, 1 - b2
        d.decay, d.step_size = 1 - lr * wd, -lr / bc1
        d.inv_sqrt_bc2, d.eps = 1.0 / math.sqrt(bc2), it["eps"]
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.mdq_fakequant_adamw_multi(arr, len(items),
                                           stream if stream is not None else _stream_handle(dev))
    _lib.check(st)
