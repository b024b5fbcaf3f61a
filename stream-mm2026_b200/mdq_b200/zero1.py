"""ZeRO-1 optimizer-state sharding for the fused MDQ step.

Replaces the reference's sharding role of DeepSpeed ZeRO-2
(CUDA/7B/llama7b_common.py:90-97) and the DDP gradient all-reduce before the
step (baseline/pretrain_gpt.py:235).  Each rank keeps the low-bit moments and
block scales of 1/world of the parameters only:

  1. gradients live in one flat buffer (``flat_grad``; ``p.grad`` are views),
     reduce-scattered (average) so each rank receives its shard;
  2. the fused step updates the rank's shard of the flat fp32 parameters;
  3. the parameters are all-gathered in place, so every rank's model sees the
     update (``p.data`` are views of ``flat_param``).

Layout.  Parameter i occupies [off_i, off_i + n_i) of the flat buffers, with
off_i a multiple of the quantisation block B and the segment padded to a whole
number of blocks, so a block never spans two parameters and a parameter's last
(partial) block keeps the reference's tail semantics (CUDA/stquant_kernel.cu:
92-97).  Parameters are grouped in order into buckets (one by default); each
bucket is padded to world * S with S a multiple of B, and rank r owns
[base + r*S, base + (r+1)*S) of every bucket.  A parameter may span ranks:
each rank holds the pieces of it that fall in its shards, cut at block
boundaries, so the sharded step computes exactly the codes, scales and
parameters of the unsharded one.  Buckets are the unit of communication: with
``overlap_grad_reduce`` a bucket's reduce-scatter starts during backward, as
soon as its last gradient is accumulated (the role DDP's bucketed all-reduce
plays in baseline/pretrain_gpt.py:235).

Bit policy.  The reference scores each tensor from torch reductions of its
full gradient (CUDA/stquant_opt_simple.py:94-98).  No rank holds a full
gradient here, so each rank sums (sum g, sum g^2, sum |g|, count) over its
pieces, the sums are all-reduced, and n_l, r_l (unbiased std / mean|g|) and v_l
follow in float64.  These agree with the reference's float32 statistics to
rounding, so a score within ~1e-6 of a threshold (24 / 12 / 6.8) can pick the
other bit width; with ``fixed_bits`` the sharded step is bit-exact.
"""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from . import kernels
from ._lib import TensorDesc
from .optim import MDQAdamWSimpleFusedIO, _zero_codes, stats_from_sums


@dataclass
class Piece:
    """Part of parameter `param` on this rank: elements [start, start + n) of
    the parameter, at `flat_off` in the flat buffers (block-aligned)."""

    param: int
    start: int
    n: int
    flat_off: int


@dataclass
class Bucket:
    """Parameters [first, last) laid out in flat elements [base, base + world*shard)."""

    first: int
    last: int
    base: int
    shard: int


class ShardLayout:
    """Block-aligned placement of parameters in flat buffers and shards.

    Parameters are grouped, in order, into buckets of about ``bucket_elems``
    elements (one bucket when None).  Each bucket is laid out on its own: every
    parameter at a block-aligned offset, the bucket padded to world * shard
    with shard a multiple of the block, rank r owning
    [base + r*shard, base + (r+1)*shard).  Buckets are the unit of the
    gradient reduce-scatter and the parameter all-gather."""

    def __init__(self, numels: List[int], block: int, world: int,
                 bucket_elems: Optional[int] = None):
        self.block = block
        self.world = world
        self.numels = list(numels)
        self.offsets = [0] * len(numels)
        self.buckets: List[Bucket] = []
        base, i = 0, 0
        while i < len(numels) or not self.buckets:
            first, off = i, 0
            while i < len(numels):
                padded = -(-numels[i] // block) * block
                if bucket_elems is not None and i > first and off + padded > bucket_elems:
                    break
                self.offsets[i] = base + off
                off += padded
                i += 1
            blocks = off // block
            shard = -(-blocks // world) * block if blocks else block
            self.buckets.append(Bucket(first, i, base, shard))
            base += shard * world
        self.total = base

    @property
    def shard(self) -> int:
        """Shard length of a one-bucket layout."""
        if len(self.buckets) != 1:
            raise AttributeError("a bucketed layout has one shard length per bucket")
        return self.buckets[0].shard

    def shard_range(self, bucket: Bucket, rank: int):
        lo = bucket.base + rank * bucket.shard
        return lo, lo + bucket.shard

    def pieces(self, rank: int) -> List[Piece]:
        out = []
        for b in self.buckets:
            lo, hi = self.shard_range(b, rank)
            for i in range(b.first, b.last):
                off, n = self.offsets[i], self.numels[i]
                a, e = max(off, lo), min(off + n, hi)
                if a < e:
                    out.append(Piece(param=i, start=a - off, n=e - a, flat_off=a))
        assert len({pc.param for pc in out}) == len(out), "one piece per parameter and rank"
        return out


class ZeroMDQAdamW(MDQAdamWSimpleFusedIO):
    """State-sharded MDQ-AdamW (FusedIO semantics per parameter piece).

    Arguments are those of the reference optimizer plus ``process_group``
    (default: the world group), ``grad_dtype`` (fp32 or bf16 flat gradients),
    ``bucket_elems`` (reduce-scatter / all-gather granularity; one bucket when
    None) and ``overlap_grad_reduce``: when set, each bucket's gradient
    reduce-scatter is launched asynchronously from a post-accumulate-grad hook
    as soon as backward has produced all of its gradients, so communication
    overlaps the rest of backward; ``step()`` waits for them.  Inside
    ``no_sync()`` (gradient accumulation) the hooks launch nothing.  The block
    is one per optimizer (``block_size``, clamped to 1024 unless
    ``exact_block``).

    ``param_dtype`` is the dtype of the model's parameters and of the
    all-gather.  float32 (default) is the reference's: the fused step updates
    the rank's shard of the fp32 parameters in place and they are
    all-gathered in fp32.  bfloat16 halves the all-gather: the model's
    parameters become bf16 views of the flat buffer, each rank keeps its
    shard's fp32 master parameters, and the step kernel itself writes the
    updated shard rounded to bf16 into the flat buffer, which is the
    all-gather's send buffer (gradients are then bf16 too).

    The all-gather runs per bucket, each started as soon as the bucket's
    step kernel is queued, so it overlaps the step of the buckets after it.
    With ``overlap_param_gather`` step() returns without waiting for them:
    call ``attach(model)`` once, and each module's forward waits (a forward
    pre-hook) for the buckets holding its own parameters, so the gathers
    overlap the next forward; ``wait_param_gather()`` waits for all.
    ``profile_phases`` records CUDA events around the reduce-scatter, the
    step kernels and the all-gather; ``last_phase_ms()`` reads them.

    ``param_gather="peer"`` (NCCL groups of up to 8 GPUs) puts the flat
    parameter buffer in symmetric memory: the step kernel stores each updated
    parameter into every rank's copy directly over NVLink (bf16 with bf16
    parameters, else fp32), so the step is its own all-gather, and one small
    all-reduce at the end orders the ranks.  "nccl" (default) all-gathers
    each bucket with NCCL after its step kernel.  ``grad_reduce="peer"``
    (with ``fixed_bits``) puts the gradients in symmetric memory too: instead
    of a reduce-scatter, the step kernel reads every rank's gradient of each
    element it owns over NVLink and averages them (fp32 sum in rank order),
    so one kernel does reduce-scatter, step and all-gather.
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                 alpha=0.9, layer_count=24, batch_size=32, update_freq=20, block_size=256,
                 *, process_group=None, grad_dtype=torch.float32, bucket_elems=None,
                 overlap_grad_reduce=False, param_dtype=torch.float32,
                 overlap_param_gather=False, profile_phases=False, param_gather="nccl",
                 grad_reduce="nccl", **kw):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                         alpha=alpha, layer_count=layer_count, batch_size=batch_size,
                         update_freq=update_freq, block_size=block_size, **kw)
        blocks = {self._block_of(g) for g in self.param_groups}
        if len(blocks) != 1:
            raise ValueError("ZeroMDQAdamW needs one block_size for all param groups")
        self.block = blocks.pop()
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.params = [p for g in self.param_groups for p in g["params"]]
        self.param_group_of = [g for g in self.param_groups for _ in g["params"]]
        for p in self.params:
            if p.dtype != torch.float32:
                raise RuntimeError("MDQ parameters must be float32")
        if param_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("param_dtype must be torch.float32 or torch.bfloat16")
        if param_dtype == torch.bfloat16:
            grad_dtype = torch.bfloat16
        self.param_dtype = param_dtype
        dev = self.params[0].device
        self.layout = ShardLayout([p.numel() for p in self.params], self.block, self.world,
                                  bucket_elems)
        self.pieces = self.layout.pieces(self.rank)
        # fp32 master parameters of this rank's shards (bf16 parameters only):
        # bucket k's shard at [master_base[k], master_base[k] + shard_k).
        self.master = None
        self.master_base = []
        if param_dtype == torch.bfloat16:
            base = 0
            for b in self.layout.buckets:
                self.master_base.append(base)
                base += b.shard
            self.master = torch.zeros(base, dtype=torch.float32, device=dev)
            for pc in self.pieces:
                mo = self._master_off(pc)
                src = self.params[pc.param].detach().reshape(-1)[pc.start:pc.start + pc.n]
                self.master[mo:mo + pc.n].copy_(src)
        if param_gather not in ("nccl", "peer"):
            raise ValueError("param_gather must be 'nccl' or 'peer'")
        self.param_gather = param_gather
        self._peer_deltas = None
        if grad_reduce not in ("nccl", "peer"):
            raise ValueError("grad_reduce must be 'nccl' or 'peer'")
        self.grad_reduce = grad_reduce
        self._grad_ranks = None
        if param_gather == "peer":
            self.flat_param, deltas = self._symmetric_flat(param_dtype, dev)
            self._peer_deltas = [d for r, d in enumerate(deltas) if r != self.rank]
        else:
            self.flat_param = torch.zeros(self.layout.total, dtype=param_dtype, device=dev)
        if grad_reduce == "peer":
            if self.fixed_bits is None:
                raise ValueError("grad_reduce='peer' needs fixed_bits: the bit policy reads the "
                                 "reduced gradients before the step")
            self.flat_grad, deltas = self._symmetric_flat(grad_dtype, dev)
            self._grad_ranks = (1.0 / self.world, deltas)
            overlap_grad_reduce = False
        else:
            self.flat_grad = torch.zeros(self.layout.total, dtype=grad_dtype, device=dev)
        for p, off in zip(self.params, self.layout.offsets):
            n = p.numel()
            self.flat_param[off:off + n].copy_(p.detach().reshape(-1))
            p.data = self.flat_param[off:off + n].view_as(p)
            if grad_dtype != p.dtype and hasattr(p, "grad_dtype"):
                p.grad_dtype = grad_dtype  # low-precision gradients of fp32 parameters
            p.grad = self.flat_grad[off:off + n].view_as(p)
        self.overlap_param_gather = bool(overlap_param_gather)
        self._ag_works = [None] * len(self.layout.buckets)
        self._module_hooks = []
        self.profile_phases = bool(profile_phases)
        self._phase_events = None
        self._descs = None
        # Asynchronous bucket reduce-scatters launched during backward.
        self._bucket_of = [0] * len(self.params)
        for k, b in enumerate(self.layout.buckets):
            for i in range(b.first, b.last):
                self._bucket_of[i] = k
        self._ready = [0] * len(self.layout.buckets)
        self._works = [None] * len(self.layout.buckets)
        self._sync = True
        self._hooks = []
        if overlap_grad_reduce and self.world > 1:
            for i, p in enumerate(self.params):
                self._hooks.append(p.register_post_accumulate_grad_hook(self._grad_ready(i)))

    # ------------------------------------------------------------------
    def zero_grad(self, set_to_none: bool = False):
        """Zero the flat gradient buffer (the views stay attached)."""
        self.flat_grad.zero_()

    @contextlib.contextmanager
    def no_sync(self):
        """Backward passes inside accumulate gradients without communication."""
        prev, self._sync = self._sync, False
        try:
            yield
        finally:
            self._sync = prev

    def _grad_ready(self, i: int):
        def hook(_p):
            if not self._sync:
                return
            k = self._bucket_of[i]
            self._ready[k] += 1
            b = self.layout.buckets[k]
            if self._ready[k] == b.last - b.first and self._works[k] is None:
                self._works[k] = self._reduce_scatter_bucket(b, async_op=True)
        return hook

    def _piece_state(self, pc: Piece):
        """State of one local piece, initialised as the reference initialises
        a tensor's state (CUDA/stquant_opt_simple.py:212-225)."""
        p = self.params[pc.param]
        st = self.state[p]
        if len(st) == 0:
            proxy = self.flat_param[pc.flat_off:pc.flat_off + pc.n]
            nb = -(-pc.n // self.block)
            st["step"] = 0
            if self.fixed_bits is None:
                st["exp_avg"] = torch.zeros(pc.n, dtype=torch.int16, device=p.device)
                st["exp_avg_sq"] = torch.zeros(pc.n, dtype=torch.uint16, device=p.device)
                st["current_bit"] = 16
            else:
                lay = kernels.layout_for_bits(*self.fixed_bits)
                st["exp_avg"], st["exp_avg_sq"] = _zero_codes(proxy, lay)
                st["current_bit"] = max(self.fixed_bits)
            st["scale_m"] = torch.zeros(nb, dtype=torch.float32, device=p.device)
            st["scale_v"] = torch.zeros(nb, dtype=torch.float32, device=p.device)
            st["v_min"] = torch.full((nb,), -20.0, dtype=torch.float32, device=p.device)
            st["last_score"] = torch.tensor(12.0, device=p.device)
            st["piece"] = (pc.start, pc.n)
        return st

    def _symmetric_flat(self, dtype, dev):
        """A flat buffer in symmetric memory (the same layout mapped on every
        rank) and the byte offsets from it to every rank's copy, in rank
        order (0 for this rank).  param_gather="peer": the step kernel stores
        each updated parameter into every rank's copy of the parameters;
        grad_reduce="peer": it sums every rank's copy of the gradients."""
        if not (dist.is_initialized() and dev.type == "cuda"
                and dist.get_backend(self.group) == "nccl"):
            raise RuntimeError("peer gathers and reductions need CUDA tensors and an NCCL "
                               "process group")
        if self.world > 8:
            raise ValueError("peer gathers and reductions support up to 8 ranks")
        import torch.distributed._symmetric_memory as symm_mem

        flat = symm_mem.empty(self.layout.total, dtype=dtype, device=dev)
        flat.zero_()
        grp = self.group if self.group is not None else dist.group.WORLD
        handle = symm_mem.rendezvous(flat, grp)
        self._symm_handles = getattr(self, "_symm_handles", []) + [handle]
        ptrs = list(handle.buffer_ptrs)
        me = ptrs[handle.rank]
        self._peer_token = torch.zeros(1, device=dev)
        return flat, [ptr - me for ptr in ptrs]

    def _master_off(self, pc: Piece) -> int:
        k = self._bucket_of_piece(pc)
        lo, _ = self.layout.shard_range(self.layout.buckets[k], self.rank)
        return self.master_base[k] + (pc.flat_off - lo)

    def _bucket_of_piece(self, pc: Piece) -> int:
        for k, b in enumerate(self.layout.buckets):
            if b.first <= pc.param < b.last:
                return k
        raise KeyError(pc.param)

    def _piece_views(self, pc: Piece):
        """(fp32 parameters the step updates, gradient) of one local piece."""
        a, e = pc.flat_off, pc.flat_off + pc.n
        if self.master is not None:
            mo = self._master_off(pc)
            return self.master[mo:mo + pc.n], self.flat_grad[a:e]
        return self.flat_param[a:e], self.flat_grad[a:e]

    def master_params(self):
        """This rank's fp32 parameters of each local piece, as
        {param index: (start within the parameter, fp32 tensor)}: the
        master copy with bf16 parameters, else views of the parameters."""
        return {pc.param: (pc.start, self._piece_views(pc)[0]) for pc in self.pieces}

    # ------------------------------------------------------------------
    def _reduce_scatter_bucket(self, b: Bucket, async_op: bool = False):
        """Average one bucket's gradients onto its shard owners (in place)."""
        full = self.flat_grad[b.base:b.base + b.shard * self.world]
        if dist.get_backend(self.group) == "nccl":
            lo, hi = self.layout.shard_range(b, self.rank)
            return dist.reduce_scatter_tensor(self.flat_grad[lo:hi], full, op=dist.ReduceOp.AVG,
                                              group=self.group, async_op=async_op)
        # gloo has no reduce-scatter: all-reduce (the average is taken once
        # the sum is complete), then every rank reads its shard.
        return dist.all_reduce(full, group=self.group, async_op=async_op)

    def _finish_bucket(self, b: Bucket):
        if dist.get_backend(self.group) != "nccl":
            self.flat_grad[b.base:b.base + b.shard * self.world].div_(self.world)

    def _reduce_scatter_grads(self):
        if self.world == 1:
            return
        for k, b in enumerate(self.layout.buckets):
            w = self._works[k]
            if w is None:
                self._reduce_scatter_bucket(b)
            else:
                w.wait()
            self._finish_bucket(b)
            self._works[k] = None
            self._ready[k] = 0

    def _all_gather_bucket(self, k: int):
        """Start the all-gather of bucket k's updated parameters (in place in
        the flat parameter buffer); the work is kept in _ag_works[k]."""
        if self.world == 1:
            return
        b = self.layout.buckets[k]
        full = self.flat_param[b.base:b.base + b.shard * self.world]
        lo, hi = self.layout.shard_range(b, self.rank)
        if dist.get_backend(self.group) == "nccl":
            w = dist.all_gather_into_tensor(full, self.flat_param[lo:hi], group=self.group,
                                            async_op=True)
        else:
            parts = list(full.chunk(self.world))
            w = dist.all_gather(parts, self.flat_param[lo:hi].clone(), group=self.group,
                                async_op=True)
        self._ag_works[k] = w

    def _wait_bucket(self, k: int):
        w = self._ag_works[k]
        if w is not None:
            self._ag_works[k] = None
            w.wait()

    def wait_param_gather(self):
        """Wait for every pending parameter all-gather (on the current stream)."""
        for k in range(len(self._ag_works)):
            self._wait_bucket(k)

    def attach(self, model: torch.nn.Module):
        """Make each module's forward wait for the all-gathers of the buckets
        that hold its own parameters (for ``overlap_param_gather``)."""
        index = {id(p): i for i, p in enumerate(self.params)}
        for mod in model.modules():
            ks = sorted({self._bucket_of[index[id(p)]] for p in mod.parameters(recurse=False)
                         if id(p) in index})
            if ks:
                def pre_hook(_m, _args, ks=ks):
                    for k in ks:
                        self._wait_bucket(k)
                self._module_hooks.append(mod.register_forward_pre_hook(pre_hook))

    @property
    def phase_events(self):
        """The latest step's four CUDA events (start, after the reduce-scatter,
        after the step kernels, end) with ``profile_phases``, else None; read
        them after the timed region to avoid a synchronisation per step."""
        return self._phase_events

    def last_phase_ms(self):
        """Device time of the latest step's phases (``profile_phases``):
        reduce_scatter (waiting for the gradient reduce-scatters), step (the
        fused step kernels, queued bucket after bucket with the all-gathers
        of earlier buckets running beside them), all_gather_tail (what of
        the all-gathers remained after the last step kernel) and total."""
        ev = self._phase_events
        if ev is None:
            return None
        ev[-1].synchronize()
        a, b, c, d = ev
        return {"reduce_scatter": a.elapsed_time(b), "step": b.elapsed_time(c),
                "all_gather_tail": c.elapsed_time(d), "total": a.elapsed_time(d)}

    def _global_grad_stats(self):
        """Per-parameter [n_l, r_l, v_l] from all-reduced partial sums."""
        sums = torch.zeros(len(self.params), 4, dtype=torch.float64,
                           device=self.flat_grad.device)
        views = [self._piece_views(pc)[1] for pc in self.pieces]
        if views and self.flat_grad.is_cuda:
            # One fused pass over every local piece (mdq_grad_stats_multi).
            # A rank holds at most one piece of each parameter (a parameter
            # lies in one bucket, and a rank's shard of a bucket is one
            # contiguous range), so the rows are copied, not summed: no
            # order-dependent floating-point accumulation.
            part = kernels.grad_stats(views)
            idx = torch.tensor([pc.param for pc in self.pieces], device=sums.device)
            sums.index_copy_(0, idx, part)
        else:
            # The same float64 sums with torch reductions (host tensors).
            for pc, g in zip(self.pieces, views):
                g64 = g.double()
                sums[pc.param, 0] += g64.sum()
                sums[pc.param, 1] += (g64 * g64).sum()
                sums[pc.param, 2] += g64.abs().sum()
                sums[pc.param, 3] += pc.n
        if self.world > 1:
            dist.all_reduce(sums, group=self.group)
        return stats_from_sums(sums)

    def _decide_bits_sharded(self):
        stats = self._global_grad_stats()
        avg = stats.mean(0)
        if self.n_ema is None:
            self.n_ema, self.r_ema, self.v_global_ema = avg[0], avg[1], avg[2]
        else:
            a = self.param_groups[0]["alpha"]
            self.n_ema = a * avg[0] + (1 - a) * self.n_ema
            self.r_ema = a * avg[1] + (1 - a) * self.r_ema
            self.v_global_ema = a * avg[2] + (1 - a) * self.v_global_ema
        tau = self.param_groups[0]["tau"]
        scores = []
        for i, p in enumerate(self.params):
            st = self.state[p]
            n_l, r_l, v_l = stats[i]
            s_t = 1.0 + (1.0 / torch.cosh(torch.tensor(st["step"] / tau, device=p.device,
                                                        dtype=torch.float32)))
            score = (7.2 + torch.log2(r_l / (self.r_ema + 1e-12))
                     + torch.log2(n_l / (self.n_ema + 1e-12)) + torch.log2(s_t)
                     + torch.log2(v_l / (self.v_global_ema + 1e-12)))
            st["last_score"] = score
            scores.append(score)
        for p, s in zip(self.params, torch.stack(scores).cpu().tolist()):
            self.state[p]["current_bit"] = self._score_to_bits(s)

    # ------------------------------------------------------------------
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self.total_steps += 1
        self.last_step_timings = {"quant_dequant_unpack_ms": 0.0, "quant_dequant_pack_ms": 0.0,
                                  "mdq_fused_io_fast_path_params": 0,
                                  "mdq_fused_io_fallback_params": 0}
        ev = None
        if self.profile_phases and self.flat_param.is_cuda:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            ev[0].record()
        # A pending all-gather of the previous step must land before the
        # parameters are touched again.
        self.wait_param_gather()
        if self.grad_reduce == "peer":
            # Every rank's gradients are complete before any step kernel
            # reads them (the kernels sum the ranks' copies themselves).
            if self.world > 1:
                dist.all_reduce(self._peer_token, group=self.group)
        else:
            self._reduce_scatter_grads()
        if ev is not None:
            ev[1].record()
        for pc in self.pieces:
            self._piece_state(pc)
        # A rank without a piece of some parameter still needs its step counter
        # and bits, which every rank derives identically.
        for p in self.params:
            st = self.state[p]
            if len(st) == 0:
                st["step"] = 0
                st["current_bit"] = 16 if self.fixed_bits is None else max(self.fixed_bits)
                st["last_score"] = torch.tensor(12.0, device=p.device)
        uf = self.param_groups[0]["update_freq"]
        if self.fixed_bits is None and ((self.total_steps % uf == 0) or self.total_steps < 5):
            self._decide_bits_sharded()

        held = {pc.param: pc for pc in self.pieces}
        device = self.flat_param.device
        # Bucket by bucket: queue the fused step of the bucket's local pieces,
        # then start its all-gather, which runs while later buckets step.
        for k, b in enumerate(self.layout.buckets):
            items, repack = [], []
            for i in range(b.first, b.last):
                p = self.params[i]
                st = self.state[p]
                if i not in held:
                    # Same step counting as the holders (FusedIO, incl. the
                    # double increment when the storage would change layout).
                    bits = int(st["current_bit"])
                    st["step"] += 1
                    st.setdefault("_layout_bits", 16 if self.fixed_bits is None else bits)
                    if self.fixed_bits is None and st["_layout_bits"] != bits:
                        st["step"] += 1
                        st["_layout_bits"] = bits
                    continue
                pc = held[i]
                pv, gv = self._piece_views(pc)
                first = len(items)
                # The shared FusedIO logic (step counting, storage align /
                # pack) runs on the piece's state; its step item then points
                # at the piece's views of the flat buffers.
                self._prepare_param(p, self.param_group_of[i], items, repack)
                for it in items[first:]:
                    it.p, it.grad = pv, gv
                    if self.master is not None:
                        a = pc.flat_off
                        it.p_bf16 = self.flat_param[a:a + pc.n]
                st["_layout_bits"] = int(st["current_bit"])
            self._launch(items, device)
            for st, bits in repack:
                self._pack_momentum_storage(st, bits)
            if self.param_gather == "nccl":
                self._all_gather_bucket(k)
        if (self.param_gather == "peer" or self.grad_reduce == "peer") and self.world > 1:
            # The step kernels wrote every rank's copy of the parameters or
            # read every rank's gradients: a collective on the stream orders
            # every rank's kernels before the parameters are read or the
            # gradients overwritten.
            dist.all_reduce(self._peer_token, group=self.group)
        if ev is not None:
            ev[2].record()
        if not self.overlap_param_gather:
            self.wait_param_gather()
        if ev is not None:
            if self.overlap_param_gather:
                self.wait_param_gather()  # (profiling: the phases need an end)
            ev[3].record()
            self._phase_events = ev
        return loss

    def load_consolidated_state_dict(self, state_dict):
        """Load an unsharded state (from ``consolidated_state_dict``, at any
        world size, or from an unsharded MDQ optimizer's ``state_dict``): each
        rank keeps the slices of codes and scales that fall in its pieces.
        Parameters themselves are restored by the caller (model state), except
        that with bf16 parameters the fp32 master shards are restored from the
        state's "master" entries when present (and the bf16 parameters set to
        their rounding and gathered)."""
        saved = state_dict["state"]
        for g, sg in zip(self.param_groups, state_dict["param_groups"]):
            for k, v in sg.items():
                if k != "params":
                    g[k] = v
        stats = state_dict.get("mdq_global_stats")
        if stats is not None:
            self.n_ema, self.r_ema = stats["n_ema"], stats["r_ema"]
            self.v_global_ema, self.total_steps = stats["v_global_ema"], stats["total_steps"]
        held = {pc.param: pc for pc in self.pieces}
        B = self.block
        self.state.clear()
        for i, p in enumerate(self.params):
            src = saved.get(i)
            if src is None:
                continue
            bits = int(src["current_bit"])
            st = self.state[p]
            st["step"] = int(src["step"])
            st["current_bit"] = bits
            st["last_score"] = torch.as_tensor(src["last_score"]).to(p.device, torch.float32)
            st["_layout_bits"] = bits
            pc = held.get(i)
            if pc is None:
                continue
            ea, easq = src["exp_avg"], src["exp_avg_sq"]
            a, n = pc.start, pc.n
            st["exp_avg"] = ea[a:a + n].to(p.device, copy=True)
            if easq.numel() == 0:
                st["exp_avg_sq"] = easq.to(p.device, copy=True)
            elif easq.numel() == ea.numel():
                st["exp_avg_sq"] = easq[a:a + n].to(p.device, copy=True)
            else:  # two v codes per byte
                if a % 2:
                    raise ValueError("nibble-packed v codes need an even block size")
                st["exp_avg_sq"] = easq[a // 2:a // 2 + (n + 1) // 2].to(p.device, copy=True)
            b0, nb = a // B, -(-n // B)
            for k in ("scale_m", "scale_v", "v_min"):
                st[k] = src[k][b0:b0 + nb].to(p.device, torch.float32, copy=True)
            st["piece"] = (a, n)
            if self.master is not None and "master" in src:
                mv = self._piece_views(pc)[0]
                mv.copy_(src["master"][a:a + n].to(mv.device))
                self.flat_param[pc.flat_off:pc.flat_off + n].copy_(mv)
        if self.master is not None and self.world > 1:
            for k in range(len(self.layout.buckets)):
                self._all_gather_bucket(k)
            self.wait_param_gather()

    # ------------------------------------------------------------------
    def consolidated_state_dict(self, dst: Optional[int] = None):
        """The unsharded per-parameter state (reference layout): pieces are
        gathered and concatenated in parameter order, on every rank (dst
        None) or on rank `dst` only (the others return None).  For large
        models use save_sharded / load_sharded, which gather nothing."""
        local = []
        for pc in self.pieces:
            st = self.state[self.params[pc.param]]
            # Transported as numpy: torch's object pickling mishandles uint16/32.
            rec = {k: (v.detach().cpu().numpy() if torch.is_tensor(v) else v)
                   for k, v in st.items() if k not in ("piece", "_layout_bits")}
            if self.master is not None:
                rec["master"] = self._piece_views(pc)[0].detach().cpu().numpy()
            local.append((pc.param, pc.start, rec))
        if self.world > 1 and dst is None:
            everything = [None] * self.world
            dist.all_gather_object(everything, local, group=self.group)
        elif self.world > 1:
            everything = [None] * self.world if self.rank == dst else None
            dist.gather_object(local, everything, dst=dist.get_global_rank(self.group, dst)
                               if self.group is not None else dst, group=self.group)
            if self.rank != dst:
                return None
        else:
            everything = [local]
        by_param = {}
        for rank_list in everything:
            for i, start, st in rank_list:
                st = {k: (torch.from_numpy(v) if hasattr(v, "dtype") and hasattr(v, "shape")
                          else v) for k, v in st.items()}
                by_param.setdefault(i, []).append((start, st))
        state = {}
        for i, parts in by_param.items():
            parts.sort(key=lambda t: t[0])
            first = parts[0][1]
            full = {k: first[k] for k in ("step", "current_bit", "last_score")}
            for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
                ts = [st[k] for _, st in parts if st[k].numel() or k != "exp_avg_sq"]
                full[k] = torch.cat(ts) if ts else first[k]
            if "master" in first:
                # bf16 parameters: the fp32 master weights (not part of the
                # reference's layout; load_consolidated_state_dict restores them)
                full["master"] = torch.cat([st["master"] for _, st in parts])
            state[i] = full
        return {"state": state,
                "param_groups": [{k: v for k, v in g.items() if k != "params"}
                                 for g in self.param_groups],
                "mdq_global_stats": {"n_ema": self.n_ema, "r_ema": self.r_ema,
                                     "v_global_ema": self.v_global_ema,
                                     "total_steps": self.total_steps}}

    # ------------------------------------------------------------------
    # Sharded checkpoints: every rank writes its own pieces, any world size
    # reads back the pieces it needs; nothing is gathered.
    # ------------------------------------------------------------------
    _CKPT_KEYS = ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min")

    def save_sharded(self, path: str) -> None:
        """Write this rank's optimizer state to ``path/rank<r>.pt`` and, from
        rank 0, ``path/manifest.pt`` (world size, block, parameter sizes,
        hyper-parameters, the policy's global statistics and every
        parameter's step / bit width / score).  With bf16 parameters each
        piece's fp32 master parameters are saved too.  Call on every rank."""
        import os

        os.makedirs(path, exist_ok=True)
        pieces = {}
        for pc in self.pieces:
            st = self.state[self.params[pc.param]]
            rec = {"start": pc.start, "n": pc.n}
            for k in self._CKPT_KEYS:
                rec[k] = st[k].detach().cpu().clone()
            if self.master is not None:
                rec["master"] = self._piece_views(pc)[0].detach().cpu().clone()
            pieces[pc.param] = rec
        torch.save({"rank": self.rank, "world": self.world, "pieces": pieces},
                   os.path.join(path, f"rank{self.rank:05d}.pt"))
        if self.rank == 0:
            scal = []
            for p in self.params:
                st = self.state[p]
                scal.append({"step": int(st.get("step", 0)),
                             "current_bit": int(st.get("current_bit", 16)),
                             "last_score": float(st["last_score"]) if "last_score" in st else 12.0,
                             "_layout_bits": st.get("_layout_bits")})
            torch.save({"format": "mdq-zero1-sharded-v1", "world": self.world,
                        "block": self.block, "numels": list(self.layout.numels),
                        "param_groups": [{k: v for k, v in g.items() if k != "params"}
                                         for g in self.param_groups],
                        "mdq_global_stats": {"n_ema": self.n_ema, "r_ema": self.r_ema,
                                             "v_global_ema": self.v_global_ema,
                                             "total_steps": self.total_steps},
                        "params": scal}, os.path.join(path, "manifest.pt"))
        if self.world > 1:
            dist.barrier(group=self.group)

    def load_sharded(self, path: str) -> None:
        """Load a checkpoint written by save_sharded at any world size: each
        rank memory-maps the saved rank files and copies the slices of codes,
        scales (and fp32 master parameters) that overlap its own pieces.  The
        model's parameters are restored by the caller, except that with bf16
        parameters the fp32 master shards come from the checkpoint when it
        holds them (and the bf16 parameters are set to their rounding)."""
        import os

        man = torch.load(os.path.join(path, "manifest.pt"), weights_only=False)
        if man.get("format") != "mdq-zero1-sharded-v1":
            raise ValueError(f"{path}: not an MDQ sharded checkpoint")
        if man["block"] != self.block or man["numels"] != list(self.layout.numels):
            raise ValueError("checkpoint block size or parameter sizes differ from this optimizer")
        for g, sg in zip(self.param_groups, man["param_groups"]):
            for k, v in sg.items():
                g[k] = v
        st_g = man["mdq_global_stats"]
        self.n_ema, self.r_ema = st_g["n_ema"], st_g["r_ema"]
        self.v_global_ema, self.total_steps = st_g["v_global_ema"], st_g["total_steps"]
        files = [torch.load(os.path.join(path, f"rank{r:05d}.pt"), mmap=True, weights_only=False)
                 for r in range(man["world"])]
        B = self.block
        self.state.clear()
        for i, p in enumerate(self.params):
            sc = man["params"][i]
            st = self.state[p]
            st["step"] = sc["step"]
            st["current_bit"] = sc["current_bit"]
            st["last_score"] = torch.tensor(sc["last_score"], dtype=torch.float32, device=p.device)
            if sc["_layout_bits"] is not None:
                st["_layout_bits"] = sc["_layout_bits"]
        for pc in self.pieces:
            p = self.params[pc.param]
            st = self.state[p]
            a, n = pc.start, pc.n
            out = {}
            for f in files:
                rec = f["pieces"].get(pc.param)
                if rec is None:
                    continue
                s0, ns = rec["start"], rec["n"]
                lo, hi = max(a, s0), min(a + n, s0 + ns)
                if lo >= hi:
                    continue
                if (lo - s0) % B or (lo - a) % B:
                    raise ValueError("piece boundaries are not block-aligned")
                if not out:
                    nb = -(-n // B)
                    easq = rec["exp_avg_sq"]
                    out["exp_avg"] = torch.empty(n, dtype=rec["exp_avg"].dtype)
                    if easq.numel() == 0:
                        out["exp_avg_sq"] = easq.clone()
                    elif easq.numel() == rec["exp_avg"].numel():
                        out["exp_avg_sq"] = torch.empty(n, dtype=easq.dtype)
                    else:
                        out["exp_avg_sq"] = torch.empty((n + 1) // 2, dtype=easq.dtype)
                    for k in ("scale_m", "scale_v", "v_min"):
                        out[k] = torch.empty(nb, dtype=torch.float32)
                    if "master" in rec:
                        out["master"] = torch.empty(n, dtype=torch.float32)
                d0, s_0, m = lo - a, lo - s0, hi - lo
                out["exp_avg"][d0:d0 + m] = rec["exp_avg"][s_0:s_0 + m]
                easq = rec["exp_avg_sq"]
                if easq.numel() == rec["exp_avg"].numel() and easq.numel():
                    out["exp_avg_sq"][d0:d0 + m] = easq[s_0:s_0 + m]
                elif easq.numel():
                    out["exp_avg_sq"][d0 // 2:(d0 + m + 1) // 2] = easq[s_0 // 2:(s_0 + m + 1) // 2]
                bd, bs, bm = d0 // B, s_0 // B, -(-m // B)
                for k in ("scale_m", "scale_v", "v_min"):
                    out[k][bd:bd + bm] = rec[k][bs:bs + bm]
                if "master" in rec and "master" in out:
                    out["master"][d0:d0 + m] = rec["master"][s_0:s_0 + m]
            if not out:
                continue  # saved before this piece had state
            for k in self._CKPT_KEYS:
                st[k] = out[k].to(p.device)
            st["piece"] = (a, n)
            if self.master is not None and "master" in out:
                mv = self._piece_views(pc)[0]
                mv.copy_(out["master"].to(mv.device))
                self.flat_param[pc.flat_off:pc.flat_off + n].copy_(mv)
        del files
        if self.master is not None and self.world > 1:
            for k in range(len(self.layout.buckets)):
                self._all_gather_bucket(k)
            self.wait_param_gather()
