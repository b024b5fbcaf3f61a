"""torch.optim-style MDQ optimizers on the fused sm_100a step.

Drop-ins for the reference classes
  MDQAdamWSimple         ruby320/STREAM-MM2026 CUDA/stquant_opt_simple.py:19-508
  MDQAdamWSimpleFusedIO  CUDA/stquant_opt_fused_io.py:16-93
  MDQAdamW               baseline/mdqbock_newhook.py:6-184 (constructor defaults
                         and ``robust_quantize``; the step is the fused one)
with the same constructor arguments, param-group keys, ``step()``, getters and
``state_dict`` layout (low-bit codes plus per-block fp32 scales).

What changes is the launch: the reference launches one kernel per parameter
with a host synchronisation on each side (stquant_opt_simple.py:242-266); here
every parameter is updated by one multi-tensor C-ABI call on the current
stream, without host synchronisation.  The host logic around the kernel -- bit
policy, state initialisation, storage alignment and packing, FusedIO's step
counting -- follows the reference line by line, so states evolve identically.

Extensions and options (reference behaviour unless noted):
  fixed_bits   int or (m_bits, v_bits): no score policy; state starts in the
               target layout.  (8, 4) uses int8 m codes + packed 4-bit v codes.
  exact_block  use block_size as given instead of min(block_size, 1024).
  p_mode       "exact" (default: the reference's IEEE divide and square root,
               parameters bit-identical; a 2000-step GPT-2 run reproduces
               the reference optimizer's losses bit for bit) or "fast"
               (hardware square root and reciprocal in the parameter update,
               about 1.5x faster; after 20 steps the parameters agree with the
               reference's within 1e-6 relative L2, tested at 2^27 and 2^30
               elements, but over thousands of steps the few-ulp differences
               can move a training run that sits on a loss plateau onto
               another trajectory).  Codes and block scales are bit-identical
               in both modes.
  grad_stats   "fused" (default): the policy's per-tensor statistics of every
               gradient come from one multi-tensor float64 pass
               (kernels.grad_stats) instead of the reference's three float32
               torch reductions per tensor; "reference": those torch
               reductions, as CUDA/stquant_opt_simple.py:94-98 runs them.  The
               two agree to float32 rounding, so only a score within about
               1e-6 of a threshold (6.8 / 12 / 24) can pick another width.
  bf16 gradients are accepted as they are (the reference requires fp32).
"""
from __future__ import annotations

import math
import time
from typing import Optional

import torch
import torch.distributed as dist
from torch.optim import Optimizer

from . import kernels
from ._lib import TensorDesc
from .kernels import (LAYOUT_M8V4, LAYOUT_PACKED4, LAYOUT_S8U8, LAYOUT_S16U16, LAYOUT_S32U32,
                      P_EXACT, P_FAST)

_KERNEL_PROF_SLOTS = 5
_PHASE_KEYS = ("mdq_kernel_dequant_ms", "mdq_kernel_adam_mv_ms", "mdq_kernel_scale_reduce_ms",
               "mdq_kernel_quant_ms", "mdq_kernel_update_p_ms")


def _parse_fixed_bits(fixed_bits):
    if fixed_bits is None:
        return None
    if isinstance(fixed_bits, int):
        fixed_bits = (fixed_bits, fixed_bits)
    mb, vb = (int(b) for b in fixed_bits)
    if mb not in (4, 8, 16, 32) or vb not in (4, 8, 16, 32):
        raise ValueError("fixed_bits must be 4, 8, 16 or 32 (or a pair of them)")
    return mb, vb


class MDQAdamWSimple(Optimizer):
    """Reference-compatible MDQ AdamW (CUDA/stquant_opt_simple.py:19)."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                 alpha=0.9, layer_count=24, batch_size=32, update_freq=20, block_size=256,
                 *, fixed_bits=None, exact_block: bool = False, p_mode: str = "exact",
                 grad_stats: str = "fused", profile_kernel: bool = False):
        # CUDA/stquant_opt_simple.py:33-44
        tau_adaptive = 300 * math.log(layer_count) * math.sqrt(batch_size)
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, alpha=alpha,
                        tau=tau_adaptive, update_freq=update_freq, block_size=block_size)
        super().__init__(params, defaults)
        self.n_ema = None
        self.r_ema = None
        self.v_global_ema = None
        self.total_steps = 0
        self.last_step_timings = {}
        if p_mode not in ("exact", "fast"):
            raise ValueError("p_mode must be 'exact' or 'fast'")
        self.p_mode = P_EXACT if p_mode == "exact" else P_FAST
        if grad_stats not in ("fused", "reference"):
            raise ValueError("grad_stats must be 'fused' or 'reference'")
        self.grad_stats = grad_stats
        self.fixed_bits = _parse_fixed_bits(fixed_bits)
        self.exact_block = bool(exact_block)
        self.profile_kernel = bool(profile_kernel)
        self._kernel_profile_buf = None
        self._kernel_profile_device = None
        self._pending_events = None
        self._descs = None

    # ------------------------------------------------------------------
    # block size, grad stats and score -> bits (stquant_opt_simple.py:93-109)
    # ------------------------------------------------------------------
    def _block_of(self, group) -> int:
        b = int(group.get("block_size", 256))
        return b if self.exact_block else min(b, 1024)  # stquant_opt_simple.py:234,415

    @staticmethod
    def _compute_grad_stats(grad: torch.Tensor) -> torch.Tensor:
        n_l = torch.sqrt(torch.mean(grad * grad))
        r_l = torch.std(grad) / (grad.abs().mean() + 1e-12)
        v_l = torch.mean(grad * grad)
        return torch.stack([n_l, r_l, v_l])

    @staticmethod
    def _score_to_bits(score) -> int:
        s = float(score.item()) if isinstance(score, torch.Tensor) else float(score)
        if s >= 24:
            return 32
        if s >= 12:
            return 16
        if s >= 6.8:
            return 8
        return 4

    # ------------------------------------------------------------------
    # storage pack / unpack / align (stquant_opt_simple.py:114-210)
    # ------------------------------------------------------------------
    @staticmethod
    def _is_momentum_packed4(state) -> bool:
        if "exp_avg" not in state or "exp_avg_sq" not in state:
            return False
        ea, easq = state["exp_avg"], state["exp_avg_sq"]
        return ea.dtype == torch.uint8 and easq.numel() == 0 and ea.numel() > 0

    @staticmethod
    def _unpack_packed4_momentum(state):
        packed = state["exp_avg"]
        m_u = (packed.to(torch.int32) & 0x0F).to(torch.int16)
        v_q = ((packed.to(torch.int32) >> 4) & 0x0F).to(torch.int32)
        state["exp_avg"] = (m_u - 8).to(torch.int8)
        state["exp_avg_sq"] = v_q.to(torch.uint8)

    @staticmethod
    def _pack_momentum_to_nibbles(state):
        ea, easq = state["exp_avg"], state["exp_avg_sq"]
        if ea.dtype != torch.int8 or easq.numel() != ea.numel():
            return
        dev = ea.device
        m_u = (ea.to(torch.int16) + 8).clamp(0, 15).to(torch.uint8)
        v_lo = easq.to(torch.int32).clamp(0, 15).to(torch.uint8)
        state["exp_avg"] = (m_u | (v_lo << 4)).to(dev)
        state["exp_avg_sq"] = torch.empty(0, dtype=torch.uint8, device=dev)

    @classmethod
    def _align_momentum_storage(cls, state, bits):
        if cls._is_momentum_packed4(state):
            cls._unpack_packed4_momentum(state)
        ea, easq = state["exp_avg"], state["exp_avg_sq"]
        if bits >= 32:
            if ea.dtype != torch.int32:
                state["exp_avg"] = ea.to(torch.int32)
            if easq.dtype != torch.uint32:
                state["exp_avg_sq"] = easq.to(torch.uint32)
            return
        if bits > 8:
            if ea.dtype == torch.int8:
                state["exp_avg"] = ea.to(torch.int16)
                state["exp_avg_sq"] = easq.to(torch.uint16)
            elif ea.dtype == torch.int32:
                state["exp_avg"] = ea.clamp(-32768, 32767).to(torch.int16)
                state["exp_avg_sq"] = easq.to(torch.int64).clamp(0, 65535).to(torch.uint16)
            elif ea.dtype != torch.int16:
                state["exp_avg"] = ea.to(torch.int16)
                state["exp_avg_sq"] = easq.to(torch.uint16)
            return
        if ea.dtype == torch.int16:
            state["exp_avg"] = ea.clamp(-128, 127).to(torch.int8)
            state["exp_avg_sq"] = easq.to(torch.int64).clamp(0, 255).to(torch.uint8)
        elif ea.dtype == torch.int32:
            state["exp_avg"] = ea.clamp(-128, 127).to(torch.int8)
            state["exp_avg_sq"] = easq.to(torch.int64).clamp(0, 255).to(torch.uint8)
        elif ea.dtype == torch.int8 and easq.numel() > 0 and easq.dtype != torch.uint8:
            state["exp_avg_sq"] = easq.to(torch.uint8)

    @classmethod
    def _pack_momentum_storage(cls, state, bits):
        ea, easq = state["exp_avg"], state["exp_avg_sq"]
        if bits <= 8:
            if ea.dtype == torch.int16:
                state["exp_avg"] = ea.clamp(-128, 127).to(torch.int8)
                state["exp_avg_sq"] = easq.to(torch.int64).clamp(0, 255).to(torch.uint8)
            elif ea.dtype == torch.int32:
                state["exp_avg"] = ea.clamp(-128, 127).to(torch.int8)
                state["exp_avg_sq"] = easq.to(torch.int64).clamp(0, 255).to(torch.uint8)
            elif ea.dtype == torch.int8 and easq.numel() > 0 and easq.dtype != torch.uint8:
                state["exp_avg_sq"] = easq.to(torch.uint8)
            if (bits == 4 and state["exp_avg"].dtype == torch.int8
                    and state["exp_avg_sq"].numel() == state["exp_avg"].numel()):
                cls._pack_momentum_to_nibbles(state)
            return
        if bits == 16:
            if ea.dtype == torch.int32:
                state["exp_avg"] = ea.clamp(-32768, 32767).to(torch.int16)
                state["exp_avg_sq"] = easq.to(torch.int64).clamp(0, 65535).to(torch.uint16)
            elif ea.dtype == torch.int8:
                state["exp_avg"] = ea.to(torch.int16)
                state["exp_avg_sq"] = easq.to(torch.uint16)
            return
        if bits >= 32:
            if ea.dtype != torch.int32:
                state["exp_avg"] = ea.to(torch.int32)
            if easq.dtype != torch.uint32:
                state["exp_avg_sq"] = easq.to(torch.uint32)

    # ------------------------------------------------------------------
    # state
    # ------------------------------------------------------------------
    def _init_state_if_needed(self, p, state, block_size):
        """CUDA/stquant_opt_simple.py:212-225 (fixed_bits: target layout)."""
        if len(state) != 0:
            return
        if p.dtype != torch.float32:
            raise RuntimeError("MDQ parameters must be float32")
        state["step"] = 0
        num_blocks = (p.numel() + block_size - 1) // block_size
        if self.fixed_bits is None:
            state["exp_avg"] = torch.zeros_like(p, dtype=torch.int16)
            state["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.uint16)
            state["current_bit"] = 16
        else:
            mb, vb = self.fixed_bits
            layout = kernels.layout_for_bits(mb, vb)
            ea, easq = _zero_codes(p, layout)
            state["exp_avg"], state["exp_avg_sq"] = ea, easq
            state["current_bit"] = max(mb, vb)
        state["scale_m"] = torch.zeros(num_blocks, dtype=torch.float32, device=p.device)
        state["scale_v"] = torch.zeros(num_blocks, dtype=torch.float32, device=p.device)
        state["v_min"] = torch.full((num_blocks,), -20.0, dtype=torch.float32, device=p.device)
        state["last_score"] = torch.tensor(12.0, device=p.device)

    def _kernel_profile_buf_for(self, device):
        if self._kernel_profile_buf is None or self._kernel_profile_device != device:
            self._kernel_profile_buf = torch.zeros(_KERNEL_PROF_SLOTS, dtype=torch.int64,
                                                   device=device)
            self._kernel_profile_device = device
        return self._kernel_profile_buf

    # ------------------------------------------------------------------
    # per-parameter launch preparation (stquant_opt_simple.py:231-280)
    # ------------------------------------------------------------------
    def _prepare_param(self, p, group, items, repack):
        """Simple: step += 1, align storage, queue the update, pack after."""
        state = self.state[p]
        bits = int(state["current_bit"])
        state["step"] += 1
        t0 = time.perf_counter()
        self._align_momentum_storage(state, bits)
        self.last_step_timings["quant_dequant_unpack_ms"] += (time.perf_counter() - t0) * 1e3
        items.append(self._item(p, group, state, bits, bits))
        repack.append((state, bits))

    def _item(self, p, group, state, m_bits, v_bits) -> kernels.StepItem:
        ea, easq = state["exp_avg"], state["exp_avg_sq"]
        layout = _layout_of_storage(ea, easq, m_bits, v_bits)
        grad = p.grad
        if not grad.is_contiguous():
            grad = grad.contiguous()
        return kernels.StepItem(
            p=p, grad=grad, exp_avg=ea, exp_avg_sq=easq if easq.numel() else None,
            scale_m=state["scale_m"], scale_v=state["scale_v"], v_min=state["v_min"],
            step=state["step"], block=self._block_of(group), lr=group["lr"],
            weight_decay=group["weight_decay"], eps=group["eps"], beta1=group["betas"][0],
            beta2=group["betas"][1], m_bits=m_bits, v_bits=v_bits, layout=layout)

    def _launch(self, items, device) -> None:
        """One C-ABI call for all queued tensors, on the current stream."""
        if not items:
            return
        if self._descs is None or len(self._descs) < len(items):
            self._descs = (TensorDesc * len(items))()
        for d, it in zip(self._descs, items):
            if not (it.p.is_cuda and it.grad.is_cuda):
                raise RuntimeError("p/grad must be CUDA")
            kernels.fill_desc(d, it)
        prof = None
        if self.profile_kernel:
            prof = self._kernel_profile_buf_for(device)
            prof.zero_()
        with torch.cuda.device(device):
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            kernels.run_descs(self._descs, len(items), device, self.p_mode, prof,
                              peer_deltas=getattr(self, "_peer_deltas", None),
                              grad_ranks=getattr(self, "_grad_ranks", None))
            end.record()
        self._pending_events = (start, end, device)

    # ------------------------------------------------------------------
    # metrics / checkpoint (stquant_opt_simple.py:227-229,321-378)
    # ------------------------------------------------------------------
    def get_last_step_timings(self):
        """Timings of the latest step() in ms (kernel time from CUDA events)."""
        self._resolve_kernel_time()
        return dict(self.last_step_timings)

    def _resolve_kernel_time(self):
        ev = self._pending_events
        if ev is None:
            return
        self._pending_events = None
        start, end, device = ev
        end.synchronize()
        kernel_ms = start.elapsed_time(end)
        t = self.last_step_timings
        t["quant_dequant_kernel_ms"] = kernel_ms
        t["mdq_fused_kernel_ms"] = kernel_ms
        t["mdq_quant_dequant_ms"] = t["mdq_unpack_ms"] + kernel_ms + t["mdq_pack_ms"]
        if self.profile_kernel and device is not None:
            cycles = self._kernel_profile_buf_for(device).double().cpu().tolist()
            total = sum(cycles)
            k_ms = [kernel_ms * c / total if total > 0 else 0.0 for c in cycles]
            for key, v in zip(_PHASE_KEYS, k_ms):
                t[key] = v
            t["mdq_kernel_phases_sum_ms"] = sum(k_ms)
            t["mdq_kernel_profile_cycles"] = cycles

    def get_bit_distribution(self):
        counts = {4: 0, 8: 0, 16: 0, 32: 0}
        num_tensors = 0
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p)
                if st and "current_bit" in st:
                    b = int(st["current_bit"])
                    counts[b] = counts.get(b, 0) + 1
                    num_tensors += 1
        if num_tensors == 0:
            return {4: 0.0, 8: 0.0, 16: 0.0, 32: 0.0}
        return {b: (c / num_tensors) * 100.0 for b, c in counts.items()}

    def get_bit_distribution_param_weighted(self):
        counts_numel = {4: 0, 8: 0, 16: 0, 32: 0}
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p)
                if st and "current_bit" in st:
                    b = int(st["current_bit"])
                    counts_numel[b] = counts_numel.get(b, 0) + p.numel()
        total = sum(counts_numel.values())
        if total == 0:
            return {4: 0.0, 8: 0.0, 16: 0.0, 32: 0.0}
        return {k: (v / total) * 100.0 for k, v in counts_numel.items()}

    def get_avg_bit_param_weighted(self):
        dist_bits = self.get_bit_distribution_param_weighted()
        return float(sum(b * (perc / 100.0) for b, perc in dist_bits.items()))

    def get_all_raw_scores(self):
        scores = []
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p)
                if st and "last_score" in st:
                    scores.append(float(st["last_score"].item()))
        return scores

    def state_dict(self):
        out = super().state_dict()
        out["mdq_global_stats"] = {
            "n_ema": self.n_ema,
            "r_ema": self.r_ema,
            "v_global_ema": self.v_global_ema,
            "total_steps": self.total_steps,
        }
        return out

    def load_state_dict(self, state_dict):
        if "mdq_global_stats" in state_dict:
            state_dict = dict(state_dict)
            stats = state_dict.pop("mdq_global_stats")
            self.n_ema = stats["n_ema"]
            self.r_ema = stats["r_ema"]
            self.v_global_ema = stats["v_global_ema"]
            self.total_steps = stats["total_steps"]
        super().load_state_dict(state_dict)
        # Optimizer.load_state_dict casts every state tensor of a floating-point
        # parameter to the parameter's dtype, codes included (uint32 codes of
        # the 32-bit layout do not even survive a float32 round trip).  The
        # reference (CUDA/stquant_opt_simple.py:371-378) inherits that cast and
        # its next step then finds float storage it cannot dispatch; here the
        # saved integer code tensors are put back as they were saved.
        saved = state_dict["state"]
        ids = [i for g in state_dict["param_groups"] for i in g["params"]]
        params = [p for g in self.param_groups for p in g["params"]]
        for pid, p in zip(ids, params):
            src, dst = saved.get(pid), self.state.get(p)
            if src is None or dst is None:
                continue
            for key in ("exp_avg", "exp_avg_sq"):
                t = src.get(key)
                if torch.is_tensor(t) and not t.dtype.is_floating_point:
                    dst[key] = t.to(p.device, copy=True)

    def dequantized_moments(self, p):
        """Float m and v of one parameter, decoded from its codes and scales."""
        return dequantize_state(self.state[p], p.numel(), self._block_of(self._group_of(p)))

    def quant_error(self, block_size=None) -> float:
        """Relative L2 quantisation error of the moments, the training script's
        metric (baseline/pretrain_gpt.py:88-104): every parameter's float
        m and v (decoded from its codes) are fake-quantised at its current bit
        width with ``robust_quantize`` (blocks of ``block_size``, default the
        group's block), and sqrt(sum |x - q(x)|^2 / (sum |x|^2 + 1e-12)) is
        returned.  The sums stay on the parameters' device; one host read."""
        num = den = None
        for group in self.param_groups:
            blk = block_size or self._block_of(group)
            for p in group["params"]:
                st = self.state.get(p)
                if not st or "exp_avg" not in st:
                    continue
                bit = int(st.get("current_bit", 32))
                m, v = self.dequantized_moments(p)
                qm = self.robust_quantize(m, bit, is_v=False, block_size=blk)
                qv = self.robust_quantize(v, bit, is_v=True, block_size=blk)
                a = (m - qm).pow(2).sum() + (v - qv).pow(2).sum()
                b = m.pow(2).sum() + v.pow(2).sum()
                num = a if num is None else num + a
                den = b if den is None else den + b
        if num is None:
            return 0.0
        return float(torch.sqrt(num / (den + 1e-12)))

    def robust_quantize(self, tensor, bits, is_v=False, block_size=2048):
        """Fake-quantise a float tensor (baseline/mdqbock_newhook.py:58-83)."""
        if bits >= 31:
            return tensor
        orig_shape = tensor.shape
        flat = tensor.flatten()
        numel = flat.numel()
        pad_len = (block_size - (numel % block_size)) % block_size
        padded = torch.nn.functional.pad(flat, (0, pad_len)) if pad_len > 0 else flat
        blocked = padded.view(-1, block_size)
        eps = 1e-12
        if is_v:
            log_v = torch.log(blocked + eps)
            v_max = log_v.max(dim=1, keepdim=True)[0]
            v_min = log_v.min(dim=1, keepdim=True)[0]
            scale = (v_max - v_min) / (2 ** bits - 1)
            q = torch.round((log_v - v_min) / (scale + eps)).clamp(0, 2 ** bits - 1)
            deq = torch.exp(q * scale + v_min)
        else:
            q_levels = 2 ** (bits - 1)
            max_val = blocked.abs().max(dim=1, keepdim=True)[0]
            scale = (max_val + eps) / (q_levels - 1)
            q = torch.round(blocked / (scale + eps)).clamp(-q_levels, q_levels - 1)
            deq = q * scale
        return deq.view(-1)[:numel].view(orig_shape)

    def _group_of(self, p):
        for g in self.param_groups:
            if any(q is p for q in g["params"]):
                return g
        raise KeyError("parameter not managed by this optimizer")

    # ------------------------------------------------------------------
    # step (stquant_opt_simple.py:383-508)
    # ------------------------------------------------------------------
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()

        self._pending_events = None
        self.total_steps += 1
        self.last_step_timings = {
            "mdq_stats_ms": 0.0,
            "mdq_bit_decision_ms": 0.0,
            "mdq_grad_stats_ms": 0.0,
            "mdq_allreduce_ms": 0.0,
            "mdq_score_bits_ms": 0.0,
            "mdq_update_decision": False,
            "mdq_update_freq": 0,
            "quant_dequant_unpack_ms": 0.0,
            "quant_dequant_kernel_ms": 0.0,
            "quant_dequant_pack_ms": 0.0,
            "mdq_fused_io_fast_path_params": 0,
            "mdq_fused_io_fallback_params": 0,
        }
        update_freq = self.param_groups[0]["update_freq"]
        update_decision = (self.total_steps % update_freq == 0) or (self.total_steps < 5)
        if self.fixed_bits is not None:
            update_decision = False
        self.last_step_timings["mdq_update_decision"] = update_decision
        self.last_step_timings["mdq_update_freq"] = update_freq

        params_with_grad = []
        for group in self.param_groups:
            b_size = self._block_of(group)
            for p in group["params"]:
                if p.grad is None:
                    continue
                params_with_grad.append((p, group))
                self._init_state_if_needed(p, self.state[p], b_size)

        if update_decision and params_with_grad:
            self._decide_bits(params_with_grad)
        else:
            for k in ("mdq_grad_stats_ms", "mdq_allreduce_ms", "mdq_score_bits_ms"):
                self.last_step_timings[k] = 0.0
            self.last_step_timings["mdq_stats_ms"] = 0.0
            self.last_step_timings["mdq_bit_decision_ms"] = 0.0
            self.last_step_timings["mdq_extra_stats_ms"] = 0.0

        items, repack = [], []
        for p, group in params_with_grad:
            self._prepare_param(p, group, items, repack)

        device = params_with_grad[0][0].device if params_with_grad else None
        self._launch(items, device)

        t1 = time.perf_counter()
        for state, bits in repack:
            self._pack_momentum_storage(state, bits)
        pack_ms = (time.perf_counter() - t1) * 1e3
        self.last_step_timings["quant_dequant_pack_ms"] += pack_ms
        t = self.last_step_timings
        t["mdq_unpack_ms"] = t["quant_dequant_unpack_ms"]
        t["mdq_pack_ms"] = t["quant_dequant_pack_ms"]
        t["mdq_fused_kernel_ms"] = 0.0
        t["mdq_quant_dequant_ms"] = t["mdq_unpack_ms"] + t["mdq_pack_ms"]
        for key in _PHASE_KEYS + ("mdq_kernel_phases_sum_ms",):
            t[key] = 0.0
        t["mdq_kernel_profile_cycles"] = []
        fast_n = int(t.get("mdq_fused_io_fast_path_params", 0))
        fall_n = int(t.get("mdq_fused_io_fallback_params", 0))
        t["mdq_fused_io_fast_path_ratio"] = (fast_n / (fast_n + fall_n)) if fast_n + fall_n else 0.0
        return loss

    def _grad_stats_all(self, params_with_grad):
        """[n_l, r_l, v_l] (float32) per parameter with a gradient."""
        if self.grad_stats == "reference":
            return [self._compute_grad_stats(p.grad) for p, _ in params_with_grad]
        # One fused pass per gradient dtype over every gradient.
        grads = [p.grad if p.grad.is_contiguous() else p.grad.contiguous()
                 for p, _ in params_with_grad]
        rows = [None] * len(grads)
        for dt in {g.dtype for g in grads}:
            idx = [i for i, g in enumerate(grads) if g.dtype == dt]
            sums = kernels.grad_stats([grads[i].reshape(-1) for i in idx])
            st = stats_from_sums(sums)
            for k, i in enumerate(idx):
                rows[i] = st[k]
        return rows

    def _decide_bits(self, params_with_grad):
        """Grad stats -> global EMA -> per-tensor score -> bits
        (CUDA/stquant_opt_simple.py:427-493).  The per-tensor arithmetic is the
        reference's; only the host reads of the scores are batched into one."""
        dev = params_with_grad[0][0].device
        _sync(dev)
        t_grad = time.perf_counter()
        all_stats = self._grad_stats_all(params_with_grad)
        _sync(dev)
        grad_stats_ms = (time.perf_counter() - t_grad) * 1e3

        stats_tensor = torch.stack(all_stats)
        avg_stats = stats_tensor.mean(dim=0)
        allreduce_ms = 0.0
        if dist.is_available() and dist.is_initialized():
            _sync(dev)
            t_ar = time.perf_counter()
            dist.all_reduce(avg_stats, op=dist.ReduceOp.SUM)
            avg_stats /= dist.get_world_size()
            _sync(dev)
            allreduce_ms = (time.perf_counter() - t_ar) * 1e3

        _sync(dev)
        t_score = time.perf_counter()
        if self.n_ema is None:
            self.n_ema = avg_stats[0]
            self.r_ema = avg_stats[1]
            self.v_global_ema = avg_stats[2]
        else:
            alpha = self.param_groups[0]["alpha"]
            self.n_ema = alpha * avg_stats[0] + (1 - alpha) * self.n_ema
            self.r_ema = alpha * avg_stats[1] + (1 - alpha) * self.r_ema
            self.v_global_ema = alpha * avg_stats[2] + (1 - alpha) * self.v_global_ema

        tau = self.param_groups[0]["tau"]
        scores = []
        for i, (p, _group) in enumerate(params_with_grad):
            state = self.state[p]
            n_l, r_l, v_l = stats_tensor[i]
            s_t = 1.0 + (1.0 / torch.cosh(
                torch.tensor(state["step"] / tau, device=p.device, dtype=torch.float32)))
            score = (7.2
                     + torch.log2(r_l / (self.r_ema + 1e-12))
                     + torch.log2(n_l / (self.n_ema + 1e-12))
                     + torch.log2(s_t)
                     + torch.log2(v_l / (self.v_global_ema + 1e-12)))
            state["last_score"] = score
            scores.append(score)
        values = torch.stack(scores).cpu().tolist()
        for (p, _group), s in zip(params_with_grad, values):
            self.state[p]["current_bit"] = self._score_to_bits(s)
        _sync(dev)
        score_bits_ms = (time.perf_counter() - t_score) * 1e3
        t = self.last_step_timings
        t["mdq_grad_stats_ms"] = grad_stats_ms
        t["mdq_allreduce_ms"] = allreduce_ms
        t["mdq_score_bits_ms"] = score_bits_ms
        t["mdq_stats_ms"] = grad_stats_ms
        t["mdq_bit_decision_ms"] = allreduce_ms + score_bits_ms
        t["mdq_extra_stats_ms"] = grad_stats_ms + allreduce_ms + score_bits_ms


class MDQAdamWSimpleFusedIO(MDQAdamWSimple):
    """CUDA/stquant_opt_fused_io.py:16: skips the Python pack/unpack when the
    storage already matches the bit width, else falls back to the Simple path
    (whose own step increment makes that step count twice, as in the
    reference, stquant_opt_fused_io.py:44-50 + stquant_opt_simple.py:236)."""

    @classmethod
    def _storage_matches_bits(cls, state, bits: int) -> bool:
        if "exp_avg" not in state:
            return False
        ea, easq = state["exp_avg"], state.get("exp_avg_sq")
        if bits == 4:
            return cls._is_momentum_packed4(state)
        if bits == 8:
            return (ea.dtype == torch.int8 and easq is not None and easq.dtype == torch.uint8
                    and easq.numel() == ea.numel())
        if bits == 16:
            return ea.dtype == torch.int16 and easq is not None and easq.dtype == torch.uint16
        if bits >= 32:
            return ea.dtype == torch.int32 and easq is not None and easq.dtype == torch.uint32
        return False

    def _prepare_param(self, p, group, items, repack):
        state = self.state[p]
        if self.fixed_bits is not None:
            # Fixed layout: the storage always matches; one increment per step.
            state["step"] += 1
            self.last_step_timings["mdq_fused_io_fast_path_params"] += 1
            items.append(self._item(p, group, state, *self.fixed_bits))
            return
        bits = int(state["current_bit"])
        state["step"] += 1
        if not self._storage_matches_bits(state, bits):
            self.last_step_timings["mdq_fused_io_fallback_params"] += 1
            return super()._prepare_param(p, group, items, repack)
        self.last_step_timings["mdq_fused_io_fast_path_params"] += 1
        items.append(self._item(p, group, state, bits, bits))


class MDQAdamW(MDQAdamWSimpleFusedIO):
    """Constructor drop-in for ``baseline/mdqbock_newhook.py:MDQAdamW`` as
    used by ``baseline/pretrain_gpt.py:192-198`` (same defaults, block 2048),
    but NOT the same algorithm: this class stores m and v as low-bit codes with
    the CUDA kernel family's semantics (CUDA/stquant_kernel.cu; block clamped
    to 1024, the FusedIO step counting), while the pure-PyTorch class keeps
    fp32 moments and only fake-quantises them for the update.  After 20 steps
    of BASELINE config 1 the two differ by about 7% relative L2 in the
    parameters.  MDQAdamWFakeQuant reproduces the pure-PyTorch class's
    algorithm.  (``robust_quantize`` and ``quant_error`` come with every
    class here.)"""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                 alpha=0.9, layer_count=12, batch_size=8, update_freq=20, block_size=2048,
                 **kw):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                         alpha=alpha, layer_count=layer_count, batch_size=batch_size,
                         update_freq=update_freq, block_size=block_size, **kw)


class MDQAdamWFakeQuant(MDQAdamWSimple):
    """The reference's pure-PyTorch MDQAdamW (baseline/mdqbock_newhook.py:6-184)
    with the same algorithm: fp32 first and second moments are kept, and each
    step updates the parameters with block-fake-quantised copies of them
    (robust_quantize at the tensor's current bit width, blocks of
    ``block_size`` -- 2048 by default, never clamped).  The score policy,
    state layout (``exp_avg`` / ``exp_avg_sq`` fp32, ``step``,
    ``current_bit``, ``last_score``, ``mdq_global_stats``) and checkpoints are
    the reference's.  What changes is the step: one fused kernel pass
    (kernels.fakequant_step, ``mdq_fakequant_adamw_multi``) per step for every
    parameter instead of about twenty torch operations per parameter.  Use
    this class to keep the reference's training dynamics exactly; MDQAdamW
    stores the moments as low-bit codes instead (about 1/4 to 1/8 of the
    optimizer memory) with the CUDA kernel family's semantics."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                 alpha=0.9, layer_count=12, batch_size=8, update_freq=20, block_size=2048,
                 *, grad_stats: str = "fused"):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                         alpha=alpha, layer_count=layer_count, batch_size=batch_size,
                         update_freq=update_freq, block_size=block_size, exact_block=True,
                         grad_stats=grad_stats)

    def _init_state_if_needed(self, p, state, block_size):
        """baseline/mdqbock_newhook.py:102-107."""
        if len(state) != 0:
            return
        if p.dtype != torch.float32:
            raise RuntimeError("MDQ parameters must be float32")
        state["step"] = 0
        state["exp_avg"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
        state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
        state["current_bit"] = 16
        state["last_score"] = torch.tensor(12.0, device=p.device)

    def dequantized_moments(self, p):
        st = self.state[p]
        return st["exp_avg"].reshape(-1), st["exp_avg_sq"].reshape(-1)

    @torch.no_grad()
    def step(self, closure=None):
        """baseline/mdqbock_newhook.py:86-175."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._pending_events = None
        self.total_steps += 1
        self.last_step_timings = {k: 0.0 for k in ("mdq_stats_ms", "mdq_bit_decision_ms",
                                                   "mdq_grad_stats_ms", "mdq_allreduce_ms",
                                                   "mdq_score_bits_ms")}
        update_decision = ((self.total_steps % self.param_groups[0]["update_freq"] == 0)
                           or (self.total_steps < 5))
        params_with_grad = []
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                params_with_grad.append((p, group))
                self._init_state_if_needed(p, self.state[p], group["block_size"])
        if update_decision and params_with_grad:
            self._decide_bits(params_with_grad)
        items = []
        for p, group in params_with_grad:
            st = self.state[p]
            st["step"] += 1
            grad = p.grad if p.grad.is_contiguous() else p.grad.contiguous()
            items.append(dict(p=p, grad=grad, exp_avg=st["exp_avg"],
                              exp_avg_sq=st["exp_avg_sq"], block=group["block_size"],
                              bits=int(st["current_bit"]), beta1=group["betas"][0],
                              beta2=group["betas"][1], lr=group["lr"],
                              weight_decay=group["weight_decay"], eps=group["eps"],
                              step=st["step"]))
        if items:
            dev = items[0]["p"].device
            with torch.cuda.device(dev):
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record()
                kernels.fakequant_step(items)
                end.record()
            self._pending_events = (start, end, None)
        t = self.last_step_timings
        for k in ("mdq_unpack_ms", "mdq_pack_ms", "quant_dequant_unpack_ms",
                  "quant_dequant_pack_ms"):
            t[k] = 0.0
        return loss


# ----------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------
def stats_from_sums(sums: torch.Tensor) -> torch.Tensor:
    """[n_l, r_l, v_l] per row (float32) from float64 rows of
    (sum g, sum g^2, sum |g|, count): n_l = sqrt(mean g^2), r_l = unbiased
    std / (mean |g| + 1e-12), v_l = mean g^2, the quantities of
    CUDA/stquant_opt_simple.py:94-98, evaluated in float64.  A one-element
    tensor has r_l = NaN, as torch.std gives it."""
    s, s2, sa, cnt = sums.unbind(1)
    mean_sq = s2 / cnt
    var = (s2 - s * s / cnt) / (cnt - 1)
    n_l = torch.sqrt(mean_sq)
    r_l = torch.sqrt(var.clamp_min(0)) / (sa / cnt + 1e-12)
    return torch.stack([n_l, r_l, mean_sq], 1).float()


def _sync(device):
    if device is not None and device.type == "cuda":
        torch.cuda.synchronize(device)


def _zero_codes(p: torch.Tensor, layout: int):
    n, dev = p.numel(), p.device
    if layout == LAYOUT_PACKED4:
        # A zero code pair is byte 0x08 (m nibble 8 = code 0, v code 0).
        return (torch.full_like(p, 8, dtype=torch.uint8),
                torch.empty(0, dtype=torch.uint8, device=dev))
    if layout == LAYOUT_S8U8:
        return torch.zeros_like(p, dtype=torch.int8), torch.zeros_like(p, dtype=torch.uint8)
    if layout == LAYOUT_S16U16:
        return torch.zeros_like(p, dtype=torch.int16), torch.zeros_like(p, dtype=torch.uint16)
    if layout == LAYOUT_S32U32:
        return torch.zeros_like(p, dtype=torch.int32), torch.zeros_like(p, dtype=torch.uint32)
    if layout == LAYOUT_M8V4:
        return (torch.zeros_like(p, dtype=torch.int8),
                torch.zeros((n + 1) // 2, dtype=torch.uint8, device=dev))
    raise ValueError(layout)


def _layout_of_storage(ea: torch.Tensor, easq: torch.Tensor, m_bits: int, v_bits: int) -> int:
    """Kernel layout of a state's storage (dispatch of CUDA/stquant_kernel.cu:430-463,
    plus the int8 + nibble-v layout of the (8, 4) extension)."""
    if ea.dtype == torch.uint8 and easq.numel() == 0:
        return LAYOUT_PACKED4
    if ea.dtype == torch.int8 and easq.dtype == torch.uint8:
        return LAYOUT_S8U8 if easq.numel() == ea.numel() else LAYOUT_M8V4
    if ea.dtype == torch.int16 and easq.dtype == torch.uint16:
        return LAYOUT_S16U16
    if ea.dtype == torch.int32 and easq.dtype == torch.uint32:
        return LAYOUT_S32U32
    raise RuntimeError(f"MDQ: unsupported state storage {ea.dtype}/{easq.dtype}")


def dequantize_state(state, n: int, block: int):
    """Float (m, v) of a state dict entry, decoded exactly as the kernel does
    before its update (m = q * scale_m, v = exp(q * scale_v + v_min))."""
    ea, easq = state["exp_avg"], state["exp_avg_sq"]
    layout = _layout_of_storage(ea, easq, 0, 0)
    if layout == LAYOUT_PACKED4:
        b = ea.to(torch.int32)
        qm, qv = (b & 15) - 8, b >> 4
    elif layout == LAYOUT_M8V4:
        qm = ea.to(torch.int32)
        pair = easq.to(torch.int32)
        qv = torch.stack([pair & 15, pair >> 4], dim=1).flatten()[:n]
    else:
        qm, qv = ea.to(torch.int64), easq.to(torch.int64)
    qm, qv = qm.flatten().float(), qv.flatten().float()
    idx = torch.arange(n, device=ea.device) // block
    m = qm * state["scale_m"][idx]
    v = torch.exp(qv * state["scale_v"][idx] + state["v_min"][idx])
    return m, v
