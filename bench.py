"""Benchmark of the fused quantized-AdamW (MDQ) step on B200.

Workload (its largest point): one flat fp32 parameter
tensor of 2^30 elements per GPU, p ~ N(0, 0.02^2), bf16 gradients
~ N(0, 1e-3^2), 4-bit m/v codes in the reference's packed layout, block 2048
requested (the reference's CUDA path clamps it to a 1024-element quantisation
block), lr 1e-3, betas (0.9, 0.999), eps 1e-8, weight decay 0.01.  A step is
one fused step over the whole tensor.  Inputs (~7.3 GB per GPU) exceed the
126 MB L2, so no flush is needed between steps.

Under torchrun each rank holds its own 2^30-element shard of the optimizer
state and steps it independently (ZeRO-1 state partitioning; the step itself
has no data-path collective), so scaling is weak and `value` is the whole
job's parameters per second: N * 2^30 / (max over ranks of the step time).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                    [--bits 4|8] [--block B] [--log2-elements k]   (other config-2 points)

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "stream-mm2026_b200"))
sys.path.insert(0, REPO)

METRIC = "fused q-AdamW step Gparams/s & HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
UNIT = "Gparams/s"
LOG2_N = 30
BLOCK_REQUESTED = 2048
BLOCK = min(BLOCK_REQUESTED, 1024)       # CUDA/stquant_opt_simple.py:234
# --log2-elements / --block change these for small profiling cases.
HP = dict(lr=1e-3, weight_decay=0.01, eps=1e-8, beta1=0.9, beta2=0.999)
# Algorithmic bytes per element: p read+write 8, bf16 grad 2, packed4 code
# read+write 2, and three fp32 scales read+written per block.
BYTES_PER_ELEM = 8 + 2 + 2 + 3 * 4 * 2 / BLOCK
BITS = 4                                 # --bits 8: int8 m / uint8 v codes (2 B read+written)
SPEC_HBM_GBS = 8000.0


def layout_name():
    return "packed 4-bit m/v" if BITS == 4 else "int8 m / uint8 v codes"


def config(n_gpus: int) -> dict:
    return {"workload": f"flat fp32 tensor 2^{LOG2_N} elts/GPU, {layout_name()}, bf16 grads, "
                        f"block {BLOCK_REQUESTED} (quantised per {BLOCK} as the reference)",
            "elements_per_gpu": 1 << LOG2_N, "bits": BITS, "block_requested": BLOCK_REQUESTED,
            "quant_block": BLOCK, "grad_dtype": "bf16", "param_dtype": "fp32",
            "parallelism": f"zero1-state-shard x{n_gpus}" if n_gpus > 1 else "single",
            "l2": f"inputs larger than L2 ({(1 << LOG2_N) * 7 / 2**30:.1f} GiB/GPU), no flush"}


def measured_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ----------------------------------------------------------------------------
# clocks sampled during the timed region
# ----------------------------------------------------------------------------
class ClockSampler:
    """SM clock and throttle reasons of one GPU, sampled every 10 ms through
    NVML while the timed region runs (reading only; nothing is set).  Falls
    back to nvidia-smi every 200 ms when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.sm, self.max_mhz, self.reasons = [], None, set()
        self._stop = threading.Event()
        self._nvml = self._handle()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _handle(self):
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            pr = torch.cuda.get_device_properties(self.index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            try:
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except pynvml.NVMLError:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            return h
        except Exception:  # noqa: BLE001 (no NVML: use nvidia-smi)
            return None

    def _sample_nvml(self):
        import pynvml

        self.sm.append(float(pynvml.nvmlDeviceGetClockInfo(self._nvml, pynvml.NVML_CLOCK_SM)))
        bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(self._nvml)
        for name, const in self.REASONS:
            if bits & getattr(pynvml, const, 0):
                self.reasons.add(name)

    def _sample_smi(self):
        out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                              "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=5).stdout.strip()
        s = [x.strip() for x in out.split(",")]
        self.sm.append(float(s[0]))
        self.max_mhz = float(s[1])
        for (name, _), val in zip(self.REASONS, s[3:7]):
            if val.lower() == "active":
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample_nvml() if self._nvml is not None else self._sample_smi()
            except Exception:  # noqa: BLE001 (a failed read is skipped)
                pass
            self._stop.wait(0.01 if self._nvml is not None else 0.2)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.sm), "source": "nvml" if self._nvml is not None else "nvidia-smi"}


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------
def make_state(n, device, seed):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    p = torch.randn(n, device=device, generator=g) * 0.02
    grad = (torch.randn(n, device=device, generator=g) * 1e-3).to(torch.bfloat16)
    nb = (n + BLOCK - 1) // BLOCK
    if BITS == 4:
        codes = (torch.full((n,), 8, dtype=torch.uint8, device=device), None)
    else:
        codes = (torch.zeros(n, dtype=torch.int8, device=device),
                 torch.zeros(n, dtype=torch.uint8, device=device))
    sm = torch.zeros(nb, device=device)
    sv = torch.zeros(nb, device=device)
    vmin = torch.full((nb,), -20.0, device=device)
    return p, grad, codes, sm, sv, vmin


def code_layout():
    from mdq_b200.kernels import LAYOUT_PACKED4, LAYOUT_S8U8

    return LAYOUT_PACKED4 if BITS == 4 else LAYOUT_S8U8


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from mdq_b200 import kernels
    from mdq_b200._lib import TensorDesc
    from mdq_b200.kernels import P_FAST, StepItem

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    n = 1 << LOG2_N
    p, grad, codes, sm, sv, vmin = make_state(n, device, seed=rank)
    item = StepItem(p=p, grad=grad, exp_avg=codes[0], exp_avg_sq=codes[1], scale_m=sm,
                    scale_v=sv, v_min=vmin, step=1, block=BLOCK, m_bits=BITS, v_bits=BITS,
                    layout=code_layout(), **HP)
    descs = (TensorDesc * 1)()
    stream = torch.cuda.current_stream(device)

    def step(t):
        item.step = t
        kernels.fill_desc(descs[0], item)
        kernels.run_descs(descs, 1, device, P_FAST, stream=stream.cuda_stream)

    t = 0
    for _ in range(args.warmup):
        t += 1
        step(t)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            t += 1
            step(t)
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    if world > 1:
        x = torch.tensor([ms], device=device)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        ms = float(x.item())
        dist.barrier()

    # Exact-parameter mode, same workload (extra figure, not the headline).
    def step_exact(tt):
        item.step = tt
        kernels.fill_desc(descs[0], item)
        kernels.run_descs(descs, 1, device, 1, stream=stream.cuda_stream)

    for _ in range(2):
        t += 1
        step_exact(t)
    start.record(stream)
    for _ in range(args.steps):
        t += 1
        step_exact(t)
    end.record(stream)
    torch.cuda.synchronize()
    ms_exact = start.elapsed_time(end) / args.steps

    if args.no_e2e:
        return ms, ms_exact, clk.summary(), None
    e2e_sec = run_e2e(args, device, p, grad, codes, sm, sv, vmin, t, "metric")
    rt_sec = run_e2e(args, device, p, grad, codes, sm, sv, vmin, t, "params")
    if world > 1:
        x = torch.tensor([e2e_sec, rt_sec], device=device, dtype=torch.float64)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        e2e_sec, rt_sec = (float(v) for v in x.tolist())
    e2e = {"value": round(world * n / e2e_sec / 1e9, 3), "unit": UNIT,
           "h2d_bytes_per_step": n * 2, "d2h_bytes_per_step": 8,
           "ms_per_step": round(e2e_sec * 1e3, 3),
           "with_parameter_download": {
               "value": round(world * n / rt_sec / 1e9, 3), "unit": UNIT,
               "h2d_bytes_per_step": n * 2, "d2h_bytes_per_step": n * 4,
               "ms_per_step": round(rt_sec * 1e3, 3)},
           "path": "mdq_b200.MDQAdamWSimpleFusedIO.step() over 16 parameter tensors (class "
                   "defaults); per step the bf16 gradients come from pinned host memory and "
                   "the step's metric (fp64 L2 norm of the updated parameters) goes back to it; "
                   "with_parameter_download also copies all fp32 parameters back; wall time"}
    del p, grad, codes, sm, sv, vmin
    torch.cuda.empty_cache()
    return ms, ms_exact, clk.summary(), e2e


def run_e2e(args, device, p, grad, codes, sm, sv, vmin, t0, download="metric"):
    """The same workload through the optimizer a user constructs
    (mdq_b200.MDQAdamWSimpleFusedIO, fixed 4- or 8-bit codes, block 2048
    requested), with host buffers: the 2^30 parameters are 16 parameter
    tensors of 2^26 elements; every step copies that step's bf16 gradients in
    from pinned host memory, calls optimizer.step(), and reads a result back
    to pinned host memory: download="metric" reads the step's metric, the
    float64 L2 norm of the updated parameters (8 bytes, as a training loop
    reads its loss; the parameters stay resident as in training);
    download="params" copies all updated fp32 parameters back.  Gradients are
    double buffered on the device, so step t+1's upload overlaps step t; the
    optimizer state stays resident.  Wall time per step."""
    import torch

    from mdq_b200 import MDQAdamWSimpleFusedIO

    del codes, sm, sv, vmin
    n = p.numel()
    chunk = 1 << 26
    nchunks = max(1, n // chunk)
    chunk = n // nchunks
    params = []
    for c in range(nchunks):
        q = torch.nn.Parameter(p[c * chunk:(c + 1) * chunk])
        q.grad_dtype = torch.bfloat16
        params.append(q)
    opt = MDQAdamWSimpleFusedIO(params, lr=HP["lr"], betas=(HP["beta1"], HP["beta2"]),
                                eps=HP["eps"], weight_decay=HP["weight_decay"],
                                block_size=BLOCK_REQUESTED, fixed_bits=BITS)
    h_grad = torch.empty(n, dtype=torch.bfloat16, pin_memory=True)
    h_grad.copy_(grad)
    if download == "params":
        h_p = torch.empty(n, dtype=torch.float32, pin_memory=True)
    else:
        h_p = torch.empty(1, dtype=torch.float64, pin_memory=True)
    bufs = [grad, torch.empty_like(grad)]
    comp = torch.cuda.current_stream(device)
    h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
    last_step = [None, None]   # step that last read each gradient buffer
    last_d2h = [None]

    def one_step(t):
        k = t % 2
        with torch.cuda.stream(h2d):
            if last_step[k] is not None:
                h2d.wait_event(last_step[k])
            bufs[k].copy_(h_grad, non_blocking=True)
            up = torch.cuda.Event()
            up.record(h2d)
        comp.wait_event(up)
        if last_d2h[0] is not None:
            comp.wait_event(last_d2h[0])     # the previous download read p
        for c, q in enumerate(params):
            q.grad = bufs[k][c * chunk:(c + 1) * chunk]
        opt.step()
        result = p if download == "params" else torch.linalg.vector_norm(p, dtype=torch.float64)
        done = torch.cuda.Event()
        done.record(comp)
        last_step[k] = done
        result.record_stream(d2h)   # read on the download stream
        with torch.cuda.stream(d2h):
            d2h.wait_event(done)
            h_p.copy_(result.reshape(-1), non_blocking=True)
            dn = torch.cuda.Event()
            dn.record(d2h)
        last_d2h[0] = dn

    t = 0
    for _ in range(max(2, args.warmup // 2)):
        t += 1
        one_step(t)
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 10))
    t_start = time.perf_counter()
    for _ in range(steps):
        t += 1
        one_step(t)
    torch.cuda.synchronize()
    sec = (time.perf_counter() - t_start) / steps
    del opt, params, bufs
    return sec


def gpt2_medium_shapes():
    """Parameter shapes of GPT-2 medium (24 layers, d=1024, 16 heads, vocab 50257,
    ctx 1024, tied embeddings): 355M parameters."""
    d, v, ctx, layers = 1024, 50257, 1024, 24
    shapes = [(v, d), (ctx, d)]
    for _ in range(layers):
        shapes += [(d,), (d,), (d, 3 * d), (3 * d,), (d, d), (d,), (d,), (d,),
                   (d, 4 * d), (4 * d,), (4 * d, d), (d,)]
    shapes += [(d,), (d,)]
    return shapes


def llama7b_shapes():
    """Parameter shapes of LLaMA-7B (32 layers, d=4096, 32 heads, SwiGLU FFN
    11008, RMSNorm, vocab 32000, untied embedding and head): 6.74B parameters."""
    d, f, v, layers = 4096, 11008, 32000, 32
    shapes = [(v, d)]
    for _ in range(layers):
        shapes += [(d,), (d, d), (d, d), (d, d), (d, d), (d,), (f, d), (f, d), (d, f)]
    shapes += [(d,), (v, d)]
    return shapes


SHARDED_MODELS = {
    # GPT-2 medium, 8-bit m / 4-bit v
    "gpt2-medium": dict(shapes=gpt2_medium_shapes, bits=(8, 4), block=256),
    # LLaMA-7B, 4-bit m / v (block 256 as the reference's
    # 7B driver, CUDA/7B/llama7b_common.py:190-197)
    "llama-7b": dict(shapes=llama7b_shapes, bits=4, block=256),
}


def _max_over_ranks(x, device, world):
    import torch
    import torch.distributed as dist

    if world == 1:
        return x
    t = torch.tensor(x, device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run_sharded(args, rank, world, device, name, param_dtype, bucket_elems, param_gather="nccl",
                grad_reduce="nccl"):
    """One ZeroMDQAdamW.step() of a fixed model on N GPUs (strong scaling:
    the model is the same at every N): bf16 gradients reduce-scattered over
    NCCL, the fused step on each rank's shard, parameters all-gathered.  The
    gradients are synthetic (written into the flat gradient buffer, as
    backward would leave them).  Device times, max over ranks; the phases
    come from CUDA events inside step() (profile_phases)."""
    import torch
    import torch.distributed as dist

    from mdq_b200.zero1 import ZeroMDQAdamW

    spec = SHARDED_MODELS[name]
    g = torch.Generator(device=device).manual_seed(1234)
    params = [torch.nn.Parameter(torch.empty(sh, device=device).normal_(0, 0.02, generator=g))
              for sh in spec["shapes"]()]
    n = sum(p.numel() for p in params)
    opt = ZeroMDQAdamW(params, lr=1e-3, weight_decay=0.01, block_size=spec["block"],
                       fixed_bits=spec["bits"], p_mode="fast", grad_dtype=torch.bfloat16,
                       param_dtype=param_dtype, bucket_elems=bucket_elems, profile_phases=True,
                       param_gather=param_gather, grad_reduce=grad_reduce)
    del params
    opt.flat_grad.normal_(0, 1e-3, generator=torch.Generator(device=device).manual_seed(rank))
    for _ in range(3):
        opt.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    steps = max(5, min(args.steps, 10))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    phases = []
    a.record()
    for _ in range(steps):
        opt.step()
        phases.append(opt.phase_events)
    b.record()
    torch.cuda.synchronize()
    total_ms = a.elapsed_time(b) / steps
    ph = {k: 0.0 for k in ("reduce_scatter", "step", "all_gather_tail")}
    for ev in phases:
        e0, e1, e2, e3 = ev
        ph["reduce_scatter"] += e0.elapsed_time(e1) / steps
        ph["step"] += e1.elapsed_time(e2) / steps
        ph["all_gather_tail"] += e2.elapsed_time(e3) / steps
    vals = _max_over_ranks([total_ms, ph["reduce_scatter"], ph["step"], ph["all_gather_tail"]],
                           device, world)
    total_ms, rs_ms, step_ms, ag_ms = vals
    total = opt.layout.total
    pbytes = 4 if param_dtype == torch.float32 else 2
    rs_bytes = (world - 1) * total // world * 2            # bf16 grads, per GPU
    ag_bytes = (world - 1) * total // world * pbytes
    out = {"model": f"{name} shapes ({n / 1e9:.3f}B params)", "params": n,
           "bits": spec["bits"], "block": spec["block"], "grad_dtype": "bf16",
           "param_dtype": "fp32" if param_dtype == torch.float32 else "bf16 (fp32 master shard)",
           "buckets": len(opt.layout.buckets), "steps": steps,
           "param_gather": ("step kernel stores into every rank's copy (symmetric memory, NVLink)"
                            if param_gather == "peer" else "NCCL all-gather per bucket"),
           "grad_reduce": ("step kernel sums every rank's gradients (symmetric memory, NVLink)"
                           if grad_reduce == "peer" else "NCCL reduce-scatter"),
           "ms_per_step": round(total_ms, 3),
           "gparams_per_s": round(n / (total_ms * 1e-3) / 1e9, 2),
           "phases_ms": {"reduce_scatter": round(rs_ms, 3), "step": round(step_ms, 3),
                         "all_gather_tail": round(ag_ms, 3)},
           "step_only_gparams_per_s": round(n / (step_ms * 1e-3) / 1e9, 2)}
    if world > 1:
        # Bus bandwidths only for phases that are a separate NCCL collective.
        out["nvlink"] = {
            "rs_bytes_per_gpu": rs_bytes, "ag_bytes_per_gpu": ag_bytes,
            "rs_busbw_gbs": (round(rs_bytes / (rs_ms * 1e-3) / 1e9, 1)
                             if grad_reduce == "nccl" and rs_ms > 0 else None),
            "ag_busbw_gbs": (round(ag_bytes / (ag_ms * 1e-3) / 1e9, 1)
                             if param_gather == "nccl" and len(opt.layout.buckets) == 1
                             and ag_ms > 0 else None)}
        if param_gather == "peer":
            # The step kernel carries the gather: bytes leaving each GPU per ms of step.
            out["nvlink"]["step_out_gbs"] = round(ag_bytes / (step_ms * 1e-3) / 1e9, 1)
    del opt
    torch.cuda.empty_cache()
    return out


def run_config1(device):
    """BASELINE config 1 on the GPU, beside the reference arm's CPU timing of
    the same workload: one fp32 2048 x 2048 tensor, fp32 gradients N(0,
    1e-3^2) per step, block 2048, 20 steps of (a) MDQAdamWFakeQuant, the
    reference's pure-PyTorch algorithm fused (fp32 moments), and (b)
    MDQAdamW, the same constructor with low-bit code state.  Each step()
    call (host policy included) is timed with CUDA events; median."""
    import torch

    from mdq_b200 import MDQAdamW, MDQAdamWFakeQuant

    n = CFG1_SHAPE[0] * CFG1_SHAPE[1]
    out = {}
    for name, cls in (("fakequant_fp32_moments", MDQAdamWFakeQuant),
                      ("codes_state", MDQAdamW)):
        torch.manual_seed(0)
        p = torch.nn.Parameter((torch.randn(*CFG1_SHAPE) * 0.02).to(device))
        opt = cls([p], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                  block_size=2048)
        gen = torch.Generator(device=device).manual_seed(0)
        grads = [torch.randn(*CFG1_SHAPE, device=device, generator=gen) * 1e-3
                 for _ in range(20)]
        times = []
        for rep in range(2):                      # the first pass warms up
            for t in range(20):
                p.grad = grads[t]
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                opt.step()
                b.record()
                b.synchronize()
                if rep:
                    times.append(a.elapsed_time(b))
        med = statistics.median(times)
        out[name] = {"ms_per_step": round(med, 4), "value": round(n / (med * 1e-3) / 1e9, 3),
                     "unit": UNIT, "bits": int(opt.state[p]["current_bit"])}
        del opt, p, grads
    out["what"] = ("config 1 (fp32 2048x2048, block 2048, 20 steps) through optimizer.step() "
                   "on one B200; median of 20 steps after 20 warm-up steps")
    return out


def nccl_busbw(world, device, nbytes=1 << 30):
    """Bus bandwidth of a plain NCCL all-gather and reduce-scatter of `nbytes`
    (bf16) in this run, the yardstick for the sharded step's collectives."""
    import torch
    import torch.distributed as dist

    if world == 1:
        return None
    n = nbytes // 2 // world * world
    full = torch.zeros(n, dtype=torch.bfloat16, device=device)
    rank = dist.get_rank()
    own = full[rank * (n // world):(rank + 1) * (n // world)]   # in place, as ZeRO uses it
    out = torch.empty(n // world, dtype=torch.bfloat16, device=device)
    res = {}
    for name in ("all_gather", "reduce_scatter"):
        def op():
            if name == "all_gather":
                dist.all_gather_into_tensor(full, own)
            else:
                dist.reduce_scatter_tensor(out, full, op=dist.ReduceOp.AVG)
        for _ in range(3):
            op()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            op()
        b.record()
        torch.cuda.synchronize()
        ms = _max_over_ranks([a.elapsed_time(b) / 10], device, world)[0]
        res[name + "_busbw_gbs"] = round((world - 1) / world * nbytes / (ms * 1e-3) / 1e9, 1)
    res["bytes"] = n * 2
    del full, out
    torch.cuda.empty_cache()
    return res


def zero1_parity(world, rank, device):
    """Sharded == unsharded, checked inside the bench run: a small model
    (awkward sizes, a parameter spanning ranks) stepped 5 times by
    ZeroMDQAdamW over NCCL and, on every rank, by the unsharded
    MDQAdamWSimpleFusedIO on the averaged gradients.  Gradients are small
    multiples of 2^-20, so the average over a power-of-two world is exact.
    Parameters, codes, scales and step counters of every local piece must be
    identical, for fixed 4-bit, fixed (8, 4) and the score policy, exact p,
    fp32 parameters; and for bf16 parameters (fp32 master) the master must
    equal the unsharded parameters and the gathered bf16 parameters their
    rounding.  Two cases gather through the step kernel's own stores into
    symmetric memory (param_gather="peer").  Returns True only if every rank
    agrees."""
    import torch
    import torch.distributed as dist

    from mdq_b200.optim import MDQAdamWSimpleFusedIO
    from mdq_b200.zero1 import ZeroMDQAdamW

    sizes = [1000, 3, (1 << 20) + 17, 256, 777, 2048, 5, 65536 * 3 + 5]

    def grads(r, t, bf16):
        gg = torch.Generator().manual_seed(1000 * t + r)
        if bf16:
            # |k| <= 15 units of 2^-12: every partial sum of up to 8 ranks is
            # exact in bfloat16, whatever order the reduction takes.
            return [torch.round(torch.randn(n, generator=gg) * 4).clamp(-15, 15) / 2 ** 12
                    for n in sizes]
        return [(torch.round(torch.randn(n, generator=gg) * 1024 * 2.0 ** (i % 3)) / 2 ** 20)
                for i, n in enumerate(sizes)]

    def params():
        gg = torch.Generator().manual_seed(0)
        return [torch.nn.Parameter((torch.randn(n, generator=gg) * 0.02).to(device))
                for n in sizes]

    ok = True
    for kw, pdt, gather in ((dict(fixed_bits=4), torch.float32, "nccl"),
                            (dict(fixed_bits=(8, 4)), torch.float32, "nccl"),
                            (dict(), torch.float32, "nccl"),
                            (dict(fixed_bits=4), torch.bfloat16, "nccl"),
                            (dict(fixed_bits=(8, 4)), torch.float32, "peer"),
                            (dict(fixed_bits=4), torch.bfloat16, "peer"),
                            (dict(fixed_bits=(8, 4)), torch.float32, "peer+grad"),
                            (dict(fixed_bits=4), torch.bfloat16, "peer+grad")):
        common = dict(lr=1e-3, weight_decay=0.01, block_size=256, p_mode="exact", **kw)
        ref = params()
        ref_opt = MDQAdamWSimpleFusedIO(ref, **common)
        mine = params()
        try:
            opt = ZeroMDQAdamW(mine, bucket_elems=400_000, param_dtype=pdt,
                               grad_dtype=torch.bfloat16 if pdt == torch.bfloat16 else torch.float32,
                               param_gather=gather.split("+")[0],
                               grad_reduce="peer" if gather.endswith("+grad") else "nccl",
                               **common)
        except (RuntimeError, ValueError):
            if gather.startswith("peer"):   # no symmetric memory on this box: nothing to check
                continue
            raise
        for t in range(1, 6):
            per = [grads(r, t, pdt == torch.bfloat16) for r in range(world)]
            opt.zero_grad()
            for i, p in enumerate(ref):
                avg = sum(pr[i] for pr in per) / world
                p.grad = avg.to(device)
                mine[i].grad.copy_(per[rank][i].to(mine[i].grad.dtype))
            ref_opt.step()
            opt.step()
        torch.cuda.synchronize()
        master = opt.master_params()
        for i, p in enumerate(ref):
            rs, st = ref_opt.state[p], opt.state[mine[i]]
            ok &= int(rs["step"]) == int(st["step"])
            if pdt == torch.float32:
                ok &= torch.equal(p.detach().view(torch.int32), mine[i].detach().view(torch.int32))
            else:
                ok &= torch.equal(p.detach().to(torch.bfloat16).view(torch.int16),
                                  mine[i].detach().view(torch.int16))
            if i not in master:
                continue
            start, mp = master[i]
            pc_n = mp.numel()
            ok &= torch.equal(p.detach().reshape(-1)[start:start + pc_n].view(torch.int32),
                              mp.view(torch.int32))
            b0, nb = start // 256, -(-pc_n // 256)
            for k in ("scale_m", "scale_v", "v_min"):
                ok &= torch.equal(rs[k][b0:b0 + nb].view(torch.int32), st[k].view(torch.int32))
            ea_r, ea = rs["exp_avg"], st["exp_avg"]
            ok &= torch.equal(ea_r.reshape(-1)[start:start + pc_n], ea)
            if rs["exp_avg_sq"].numel() == rs["exp_avg"].numel():
                ok &= torch.equal(rs["exp_avg_sq"].reshape(-1)[start:start + pc_n],
                                  st["exp_avg_sq"])
            elif rs["exp_avg_sq"].numel():
                ok &= torch.equal(rs["exp_avg_sq"][start // 2:start // 2 + (pc_n + 1) // 2],
                                  st["exp_avg_sq"])
        del opt, ref_opt
    flag = torch.tensor([1 if ok else 0], device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


def traffic_per_launch(n_elems):
    """DRAM bytes per launch from the committed ncu summary of this kernel,
    scaled from its capture size to this launch (traffic is proportional)."""
    lay = "packed4" if BITS == 4 else "s8u8"
    # int8/uint8 codes at 128..1024-element blocks and packed 4-bit codes at
    # 128-element blocks run the staged kernel (fast p).
    staged = (BITS == 8 and BLOCK in (128, 256, 512, 1024)) or (BITS == 4 and BLOCK == 128)
    kern = "mdq_step_staged" if staged else "mdq_step_tiles"
    path = os.path.join(REPO, "profiles", f"{kern}_{lay}_bf16_b{BLOCK}.json")
    full = os.path.join(REPO, "profiles", f"{kern}_{lay}_bf16_b{BLOCK}_2e{LOG2_N}.json")
    if os.path.exists(full):
        path = full          # a capture of this very launch size
    try:
        with open(path) as f:
            d = json.load(f)
        per_elem = (d["dram_bytes_read"] + d["dram_bytes_write"]) / d["elements"]
        return round(per_elem * n_elems), d.get("capture", "")
    except (OSError, KeyError, ValueError, ZeroDivisionError):
        return None, None


# ----------------------------------------------------------------------------
# CPU baselines (reference arm and the cpu_baseline leg)
# ----------------------------------------------------------------------------
REF_DIR = os.path.join(REPO, "oracle", "_ref")
CFG1_SHAPE = (2048, 2048)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reference_cpu_baseline(budget_s=12.0, min_steps=20):
    """The reference's own pure-PyTorch quantized AdamW
    (baseline/mdqbock_newhook.py:MDQAdamW, imported unmodified from its
    byte-compiled copy in oracle/_ref) at BASELINE config 1: one fp32
    2048 x 2048 tensor ~ N(0, 0.02^2), fp32 gradients N(0, 1e-3^2) drawn per
    step from a generator seeded 0, lr 1e-3, betas (0.9, 0.999), eps 1e-8,
    weight decay 0.01, block 2048 (the policy picks 8-bit m/v for a single
    tensor), on every host core.  Runs 20-step trajectories until `budget_s`
    and reports the median step.  None when the reference module is absent."""
    import torch

    from oracle import build_ref

    try:
        MDQAdamW = build_ref.load_python_module("mdqbock_newhook").MDQAdamW  # unmodified
    except FileNotFoundError:
        return None

    cores = host_cores()
    torch.set_num_threads(cores)
    n = CFG1_SHAPE[0] * CFG1_SHAPE[1]
    times, bits, runs = [], set(), 0
    t_all = time.perf_counter()
    while runs == 0 or (time.perf_counter() - t_all < budget_s and runs < 50):
        runs += 1
        torch.manual_seed(0)
        p = torch.nn.Parameter(torch.randn(*CFG1_SHAPE) * 0.02)
        opt = MDQAdamW([p], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                       block_size=2048)
        gen = torch.Generator().manual_seed(0)
        for _ in range(min_steps):
            p.grad = torch.randn(*CFG1_SHAPE, generator=gen) * 1e-3
            t0 = time.perf_counter()
            opt.step()
            times.append(time.perf_counter() - t0)
        bits.add(int(opt.state[p]["current_bit"]))
    med = statistics.median(times)
    return {"value": round(n / med / 1e9, 5), "unit": UNIT, "cores": cores, "kind": "reference",
            "ms_per_step": round(med * 1e3, 3),
            "sample": f"baseline/mdqbock_newhook.py MDQAdamW (pure PyTorch, unmodified) at "
                      f"config 1: fp32 2048x2048, block 2048, {sorted(bits)}-bit m/v chosen by "
                      f"its policy; median of {len(times)} step() calls ({runs} runs of "
                      f"{min_steps} steps), torch.set_num_threads({cores})"}


def port_cpu_baseline(budget_s=8.0, threads=None):
    """Second leg: the C restatement of the reference CUDA kernel
    (oracle/mdq_oracle.c) at config 1's size and 8-bit codes, block 2048
    clamped to the reference CUDA path's 1024, on `threads` host threads."""
    import numpy as np

    from oracle import oracle

    oracle.build()
    threads = threads or oracle.max_threads()
    n = CFG1_SHAPE[0] * CFG1_SHAPE[1]
    blk = 1024
    rng = np.random.default_rng(0)
    p = (rng.standard_normal(n) * 0.02).astype(np.float32)
    g = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    codes, vcodes = np.zeros(n, np.int8), np.zeros(n, np.uint8)
    nb = n // blk
    sm = np.zeros(nb, np.float32)
    sv = np.zeros(nb, np.float32)
    vmin = np.full(nb, -20.0, np.float32)
    steps = 0
    t0 = time.perf_counter()
    while True:
        steps += 1
        oracle.step(p, g, oracle.LAYOUT_S8U8, codes, vcodes, sm, sv, vmin, blk, HP["beta1"],
                    HP["beta2"], HP["lr"], HP["weight_decay"], HP["eps"], steps, 8, 8,
                    threads=threads)
        t = time.perf_counter() - t0
        if (t >= budget_s and steps >= 3) or steps >= 2000:
            break
    return {"value": round(n * steps / t / 1e9, 4), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"{steps} steps x 2^22 elements of oracle/mdq_oracle.c (C restatement of "
                      f"CUDA/stquant_kernel.cu), int8/uint8 codes, block 1024, fp32 grads, "
                      f"in {t:.1f} s"}


def cpu_baseline(budget_s=12.0):
    ref = reference_cpu_baseline(budget_s)
    port = port_cpu_baseline(budget_s=max(3.0, budget_s / 2))
    if ref is None:
        port["note"] = "reference module not built into oracle/_ref; the port stands in"
        return port
    ref["port_leg"] = port
    return ref


def run_reference_arm(args, rank, world):
    if rank != 0:
        return 0
    budget = max(5.0, min(60.0, 0.5 * (args.steps + args.warmup)))
    base = reference_cpu_baseline(budget_s=budget)
    if base is None:
        base = port_cpu_baseline(budget_s=budget)
        base["note"] = "reference module not built into oracle/_ref; the port stands in"
    n = CFG1_SHAPE[0] * CFG1_SHAPE[1]
    line = {"metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(n / (base["value"] * 1e9) * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": config(world), "impl": "reference",
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mdq_b200", choices=["mdq_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the ZeRO-1 runs of the GPT-2-medium / LLaMA-7B shapes")
    ap.add_argument("--log2-elements", type=int, default=30,
                    help="elements per GPU = 2^k (profiling cases use smaller k)")
    ap.add_argument("--block", type=int, default=2048,
                    help="requested block; quantised per min(block, 1024) as the reference")
    ap.add_argument("--bits", type=int, default=4, choices=[4, 8],
                    help="code width of m and v (4: packed layout, 8: int8 / uint8)")
    args = ap.parse_args()
    global LOG2_N, BLOCK_REQUESTED, BLOCK, BYTES_PER_ELEM, BITS
    LOG2_N, BLOCK_REQUESTED, BITS = args.log2_elements, args.block, args.bits
    BLOCK = min(BLOCK_REQUESTED, 1024)
    BYTES_PER_ELEM = 8 + 2 + (2 if BITS == 4 else 4) + 3 * 4 * 2 / BLOCK
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist

    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    ms, ms_exact, clocks, e2e = run_ours(args, rank, world, local_rank)
    dev = torch.device("cuda", local_rank)
    zero1 = None
    if not args.no_sharded:
        zero1 = {"what": "ZeroMDQAdamW.step() of fixed models (strong scaling): reduce-scatter "
                         "(avg) of bf16 gradients, fused step on each rank's shard, all-gather of "
                         "the parameters; device time, max over ranks",
                 "runs": []}
        for name in ("gpt2-medium", "llama-7b"):
            zero1["runs"].append(run_sharded(args, rank, world, dev, name, torch.float32, None))
            if world > 1:
                zero1["runs"].append(run_sharded(args, rank, world, dev, name, torch.bfloat16,
                                                 1 << 28))
                for pdt, gr in ((torch.bfloat16, "nccl"), (torch.float32, "nccl"),
                                (torch.bfloat16, "peer")):
                    try:
                        zero1["runs"].append(run_sharded(args, rank, world, dev, name, pdt, None,
                                                         param_gather="peer", grad_reduce=gr))
                    except (RuntimeError, ValueError) as e:   # no symmetric memory here
                        torch.cuda.empty_cache()
                        zero1["runs"].append({"model": name, "param_gather": "peer",
                                              "unavailable": str(e)[:300]})
        zero1["nccl_reference"] = nccl_busbw(world, dev)
        if world > 1:
            zero1["zero1_parity"] = zero1_parity(world, rank, dev)
    n = 1 << LOG2_N
    value = world * n / (ms * 1e-3) / 1e9
    bytes_launch = n * BYTES_PER_ELEM
    achieved = bytes_launch / (ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    traffic, capture = traffic_per_launch(n)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": config(world),
            "hbm_gbs_per_gpu": round(achieved, 1),
            "pct_of_8tbs": round(100 * achieved / SPEC_HBM_GBS, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": peak_kind, "traffic": traffic,
                         "traffic_source": capture,
                         "algorithmic_bytes_per_launch": round(bytes_launch)},
            "exact_p_mode": {"value": round(world * n / (ms_exact * 1e-3) / 1e9, 2),
                             "ms_per_step": round(ms_exact, 4)},
            "e2e": e2e, "gpu_launches": args.steps, "clocks": clocks,
        }
        if zero1 is not None:
            line["zero1"] = zero1
            if "zero1_parity" in zero1:
                line["zero1_parity"] = zero1["zero1_parity"]
        if world == 1 and not args.no_cpu_baseline:
            line["config1"] = run_config1(torch.device("cuda", local_rank))
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
