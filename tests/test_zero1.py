"""ZeRO-1 sharding on CPU ranks (gloo): the sharded step equals the unsharded
one.  The CUDA launch is replaced by the CPU oracle (a test double swapped in
with monkeypatch inside each rank) in both the sharded and the unsharded run;
what is under test is the partitioning, the collectives, the per-piece state
and the step counting."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mdq_b200.zero1 import ShardLayout

SIZES = [1000, 3, 4096 + 17, 256, 777, 2048, 1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _grads(rank, step, sizes):
    # Multiples of 2^-20 well inside float range: any summation order is exact.
    g = torch.Generator().manual_seed(1000 * step + rank)
    out = []
    for i, n in enumerate(sizes):
        scale = 4.0 ** (i % 4)
        out.append(torch.round(torch.randn(n, generator=g) * 1024 * scale) / 2 ** 20)
    return out


def _params(sizes):
    g = torch.Generator().manual_seed(0)
    return [torch.nn.Parameter(torch.randn(n, generator=g) * 0.02) for n in sizes]


def _use_oracle():
    import test_host_parity
    from mdq_b200 import optim

    optim.MDQAdamWSimple._launch = test_host_parity.oracle_launch
    optim.MDQAdamWSimple._grad_stats_all = test_host_parity.cpu_fused_stats


def _unsharded(world, steps, kw, sizes):
    _use_oracle()
    from mdq_b200.optim import MDQAdamWSimpleFusedIO

    torch.set_num_threads(1)
    params = _params(sizes)
    opt = MDQAdamWSimpleFusedIO([{"params": params[:4]}, {"params": params[4:], "weight_decay": 0.0}],
                                lr=1e-3, weight_decay=0.01, block_size=256, **kw)
    for t in range(1, steps + 1):
        per_rank = [_grads(r, t, sizes) for r in range(world)]
        for i, p in enumerate(params):
            p.grad = sum(pr[i] for pr in per_rank) / world
        opt.step()
    return params, opt


def _worker(rank, world, port, steps, kw, sizes, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _use_oracle()
        from mdq_b200.zero1 import ZeroMDQAdamW

        torch.set_num_threads(1)
        params = _params(sizes)
        opt = ZeroMDQAdamW([{"params": params[:4]}, {"params": params[4:], "weight_decay": 0.0}],
                           lr=1e-3, weight_decay=0.01, block_size=256, **kw)
        for t in range(1, steps + 1):
            opt.zero_grad()
            for p, g in zip(params, _grads(rank, t, sizes)):
                p.grad.copy_(g)
            opt.step()
        sd = opt.consolidated_state_dict()
        if rank == 0:
            q.put(([p.detach().numpy().copy() for p in params],
                   {i: {k: (v.numpy() if torch.is_tensor(v) else v) for k, v in st.items()}
                    for i, st in sd["state"].items()}))
    finally:
        dist.destroy_process_group()


def _run_sharded(world, steps, kw, sizes):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, steps, kw, sizes, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("bucket_elems", [None, 1, 3000])
def test_layout_is_block_aligned_and_covers_every_element(bucket_elems):
    for world in (1, 2, 3, 8):
        lay = ShardLayout(SIZES, 256, world, bucket_elems)
        assert lay.total % (world * 256) == 0
        if bucket_elems == 1:
            assert len(lay.buckets) == len(SIZES)
        seen = {i: 0 for i in range(len(SIZES))}
        for r in range(world):
            for pc in lay.pieces(r):
                assert pc.flat_off % 256 == 0 and pc.start % 256 == 0
                b = next(b for b in lay.buckets if b.first <= pc.param < b.last)
                lo, hi = lay.shard_range(b, r)
                assert lo <= pc.flat_off and pc.flat_off + pc.n <= hi
                seen[pc.param] += pc.n
        assert [seen[i] for i in range(len(SIZES))] == SIZES


@pytest.mark.parametrize("world,kw", [(2, dict(fixed_bits=(8, 4))), (4, dict(fixed_bits=16)),
                                      (3, dict())])
def test_sharded_step_equals_unsharded(world, kw):
    """Fixed bit widths (incl. the mixed layout) and the score policy, whose
    decisions here sit far from the thresholds, so float64 partial sums pick
    the same widths as the reference's float32 statistics."""
    steps = 5
    # The policy case leaves out the one-element tensor: its std is NaN,
    # which would turn every score NaN and every width to 4 bits.
    sizes = SIZES if kw else [n for n in SIZES if n > 1]
    ref_params, ref_opt = _unsharded(world, steps, kw, sizes)
    params, state = _run_sharded(world, steps, kw, sizes)
    if not kw:
        assert len({int(ref_opt.state[p]["current_bit"]) for p in ref_params}) > 1
    for i, (a, b) in enumerate(zip(ref_params, params)):
        np.testing.assert_array_equal(a.detach().numpy().view(np.int32), b.view(np.int32),
                                      err_msg=f"param {i}")
    for i, p in enumerate(ref_params):
        rs = ref_opt.state[p]
        st = state[i]
        assert st["step"] == rs["step"], i
        assert st["current_bit"] == rs["current_bit"], i
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            a = rs[k].numpy()
            np.testing.assert_array_equal(a.view(np.uint8), st[k].view(np.uint8),
                                          err_msg=f"param {i} {k}")


def _resume_worker(rank, world, port, sizes, kw, phase, payload, q):
    """Phase "save": steps 1-6, then rank 0 returns params + consolidated
    state.  Phase "resume": load them (at this world size) and run steps 7-11.
    Every rank sees the same gradients, so the result is world-independent."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _use_oracle()
        from mdq_b200.zero1 import ZeroMDQAdamW

        torch.set_num_threads(1)
        params = _params(sizes)
        if phase == "resume":
            for p, v in zip(params, payload[0]):
                p.data.copy_(torch.from_numpy(v))
        opt = ZeroMDQAdamW([{"params": params[:4]}, {"params": params[4:], "weight_decay": 0.0}],
                           lr=1e-3, weight_decay=0.01, block_size=256, **kw)
        steps = range(1, 7)
        if phase == "resume":
            if isinstance(payload[1], str):
                opt.load_sharded(payload[1])
            else:
                opt.load_consolidated_state_dict(_torch_tree(payload[1]))
            steps = range(7, 12)
        for t in steps:
            opt.zero_grad()
            for p, g in zip(params, _grads(0, t, sizes)):
                p.grad.copy_(g)
            opt.step()
        if phase == "save_sharded":
            opt.save_sharded(payload)
            sd = None
        else:
            sd = _np_tree(opt.consolidated_state_dict(dst=0))
        if rank == 0:
            q.put(([p.detach().numpy().copy() for p in params], sd))
    finally:
        dist.destroy_process_group()


def _np_tree(x):
    # Queues pickle tensors through torch's sharing path, which mishandles
    # uint16/uint32 storage; states travel as numpy.
    if torch.is_tensor(x):
        return ("__t", x.detach().cpu().numpy())
    if isinstance(x, dict):
        return {k: _np_tree(v) for k, v in x.items()}
    if isinstance(x, list):
        return [_np_tree(v) for v in x]
    return x


def _torch_tree(x):
    if isinstance(x, tuple) and len(x) == 2 and x[0] == "__t":
        return torch.from_numpy(x[1])
    if isinstance(x, dict):
        return {k: _torch_tree(v) for k, v in x.items()}
    if isinstance(x, list):
        return [_torch_tree(v) for v in x]
    return x


def _spawn(world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_resume_worker, args=(r, world, port) + args + (q,))
             for r in range(world)]
    for p in procs:
        p.start()
    out = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("w_save,w_resume,kw", [(2, 3, dict(fixed_bits=(8, 4))), (3, 2, dict())])
def test_checkpoint_resharding_resume(w_save, w_resume, kw):
    """Save a consolidated state at one world size, resume at another: the
    continued run equals an unsharded run of all eleven steps bit for bit."""
    sizes = SIZES if kw else [n for n in SIZES if n > 1]
    ref_params, ref_opt = _unsharded(1, 11, kw, sizes)
    saved = _spawn(w_save, sizes, kw, "save", None)
    params, sd = _spawn(w_resume, sizes, kw, "resume", saved)
    sd = _torch_tree(sd)
    for i, (a, b) in enumerate(zip(ref_params, params)):
        np.testing.assert_array_equal(a.detach().numpy().view(np.int32), b.view(np.int32),
                                      err_msg=f"param {i}")
    for i, p in enumerate(ref_params):
        rs, st = ref_opt.state[p], sd["state"][i]
        assert st["step"] == rs["step"] and st["current_bit"] == rs["current_bit"], i
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            np.testing.assert_array_equal(rs[k].numpy().view(np.uint8),
                                          st[k].numpy().view(np.uint8), err_msg=f"param {i} {k}")


def _overlap_worker(rank, world, port, steps, kw, sizes, q):
    """Gradients from real backward passes (loss = sum_i <p_i, c_i>, so the
    gradient is exactly c_i): two micro-batches per step, the first inside
    no_sync(); bucket reduce-scatters launched from the hooks."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _use_oracle()
        from mdq_b200.zero1 import ZeroMDQAdamW

        torch.set_num_threads(1)
        params = _params(sizes)
        opt = ZeroMDQAdamW([{"params": params[:4]}, {"params": params[4:], "weight_decay": 0.0}],
                           lr=1e-3, weight_decay=0.01, block_size=256, bucket_elems=3000,
                           overlap_grad_reduce=True, **kw)
        assert len(opt.layout.buckets) > 2
        for t in range(1, steps + 1):
            opt.zero_grad()
            coef = _grads(rank, t, sizes)
            with opt.no_sync():
                sum((p * (c / 2)).sum() for p, c in zip(params, coef)).backward()
            assert all(w is None for w in opt._works)
            sum((p * (c / 2)).sum() for p, c in zip(params, coef)).backward()
            assert all(w is not None for w in opt._works)  # launched during backward
            opt.step()
        sd = opt.consolidated_state_dict()
        if rank == 0:
            q.put(([p.detach().numpy().copy() for p in params],
                   {i: {k: (v.numpy() if torch.is_tensor(v) else v) for k, v in st.items()}
                    for i, st in sd["state"].items()}))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,kw", [(2, dict(fixed_bits=(8, 4))), (3, dict())])
def test_bucketed_overlap_equals_unsharded(world, kw):
    steps = 4
    sizes = SIZES if kw else [n for n in SIZES if n > 1]
    ref_params, ref_opt = _unsharded(world, steps, kw, sizes)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_overlap_worker, args=(r, world, port, steps, kw, sizes, q))
             for r in range(world)]
    for p in procs:
        p.start()
    params, state = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for i, (a, b) in enumerate(zip(ref_params, params)):
        np.testing.assert_array_equal(a.detach().numpy().view(np.int32), b.view(np.int32),
                                      err_msg=f"param {i}")
    for i, p in enumerate(ref_params):
        rs, st = ref_opt.state[p], state[i]
        assert st["step"] == rs["step"] and st["current_bit"] == rs["current_bit"], i
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            np.testing.assert_array_equal(rs[k].numpy().view(np.uint8), st[k].view(np.uint8),
                                          err_msg=f"param {i} {k}")


class _Term(torch.nn.Module):
    """One parameter and its loss term <p, c> (a module, so ZeroMDQAdamW.attach
    can put a forward pre-hook on it)."""

    def __init__(self, p):
        super().__init__()
        self.p = p

    def forward(self, c):
        return (self.p * c).sum()


def _bf16_grads(rank, step, sizes):
    # Small multiples of 2^-12: every value, sum over two ranks and average is
    # exact in bfloat16, so gloo's bf16 reduction matches the reference's.
    g = torch.Generator().manual_seed(1000 * step + rank)
    return [torch.round(torch.randn(n, generator=g) * 8).clamp(-31, 31) / 2 ** 12 for n in sizes]


def _bf16_worker(rank, world, port, steps, kw, sizes, q):
    """bf16 parameters, fp32 master shards, bucketed all-gathers left running
    after step() and waited for by the next forward's pre-hooks."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _use_oracle()
        from mdq_b200.zero1 import ZeroMDQAdamW

        torch.set_num_threads(1)
        params = _params(sizes)
        model = torch.nn.ModuleList([_Term(p) for p in params])
        opt = ZeroMDQAdamW([{"params": params[:4]}, {"params": params[4:], "weight_decay": 0.0}],
                           lr=1e-3, weight_decay=0.01, block_size=256, bucket_elems=3000,
                           param_dtype=torch.bfloat16, overlap_param_gather=True, **kw)
        opt.attach(model)
        assert all(p.dtype == torch.bfloat16 for p in params)
        assert len(opt.layout.buckets) > 2
        for t in range(1, steps + 1):
            opt.zero_grad()
            coef = [c.to(torch.bfloat16) for c in _bf16_grads(rank, t, sizes)]
            sum(m(c) for m, c in zip(model, coef)).backward()
            opt.step()
            if t < steps:
                assert any(w is not None for w in opt._ag_works)  # still in flight
        model[0](torch.zeros_like(params[0]))  # a forward waits for its bucket
        opt.wait_param_gather()
        masters = [None] * world
        local = {i: (s, m.numpy().copy()) for i, (s, m) in opt.master_params().items()}
        dist.all_gather_object(masters, local)
        sd = opt.consolidated_state_dict()
        if rank == 0:
            full = [np.zeros(n, np.float32) for n in sizes]
            for part in masters:
                for i, (s, m) in part.items():
                    full[i][s:s + m.size] = m
            q.put(([p.detach().float().numpy().copy() for p in params], full,
                   {i: {k: (v.numpy() if torch.is_tensor(v) else v) for k, v in st.items()}
                    for i, st in sd["state"].items()}))
    finally:
        dist.destroy_process_group()


def test_bf16_params_fp32_master_overlapped_gather():
    """bf16 model parameters: every rank's parameters are the bf16 rounding of
    the fp32 master weights, and those equal the unsharded fp32 run's
    parameters bit for bit (as do codes and scales)."""
    world, steps, kw = 2, 4, dict(fixed_bits=(8, 4))
    sizes = SIZES
    _use_oracle()
    from mdq_b200.optim import MDQAdamWSimpleFusedIO

    torch.set_num_threads(1)
    ref_params = _params(sizes)
    ref_opt = MDQAdamWSimpleFusedIO([{"params": ref_params[:4]},
                                     {"params": ref_params[4:], "weight_decay": 0.0}],
                                    lr=1e-3, weight_decay=0.01, block_size=256, **kw)
    for t in range(1, steps + 1):
        per_rank = [_bf16_grads(r, t, sizes) for r in range(world)]
        for i, p in enumerate(ref_params):
            p.grad_dtype = torch.bfloat16
            p.grad = (sum(pr[i] for pr in per_rank) / world).to(torch.bfloat16)
        ref_opt.step()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bf16_worker, args=(r, world, port, steps, kw, sizes, q))
             for r in range(world)]
    for p in procs:
        p.start()
    model_params, masters, state = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for i, p in enumerate(ref_params):
        want = p.detach().numpy()
        np.testing.assert_array_equal(masters[i].view(np.int32), want.view(np.int32),
                                      err_msg=f"master {i}")
        np.testing.assert_array_equal(model_params[i],
                                      p.detach().to(torch.bfloat16).float().numpy(),
                                      err_msg=f"bf16 param {i}")
        rs, st = ref_opt.state[p], state[i]
        assert st["step"] == rs["step"], i
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            np.testing.assert_array_equal(rs[k].numpy().view(np.uint8), st[k].view(np.uint8),
                                          err_msg=f"param {i} {k}")


def test_sharded_checkpoint_resume_at_other_world_size(tmp_path):
    """save_sharded at 2 ranks after 6 steps, load_sharded at 3 ranks and run
    5 more: equal to an unsharded 11-step run bit for bit."""
    kw = dict(fixed_bits=(8, 4))
    sizes = SIZES
    ref_params, ref_opt = _unsharded(1, 11, kw, sizes)
    ck = str(tmp_path / "ck")
    saved_params, _ = _spawn(2, sizes, kw, "save_sharded", ck)
    params, sd = _spawn(3, sizes, kw, "resume", (saved_params, ck))
    sd = _torch_tree(sd)
    for i, (a, b) in enumerate(zip(ref_params, params)):
        np.testing.assert_array_equal(a.detach().numpy().view(np.int32), b.view(np.int32),
                                      err_msg=f"param {i}")
    for i, p in enumerate(ref_params):
        rs, st = ref_opt.state[p], sd["state"][i]
        assert st["step"] == rs["step"] and st["current_bit"] == rs["current_bit"], i
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            np.testing.assert_array_equal(rs[k].numpy().view(np.uint8),
                                          st[k].numpy().view(np.uint8), err_msg=f"param {i} {k}")


def _reconstruct(path):
    """Full per-parameter codes and scales from a sharded checkpoint."""
    man = torch.load(os.path.join(path, "manifest.pt"), weights_only=False)
    B = man["block"]
    parts = {}
    for r in range(man["world"]):
        f = torch.load(os.path.join(path, f"rank{r:05d}.pt"), mmap=True, weights_only=False)
        for i, rec in f["pieces"].items():
            parts.setdefault(i, []).append(rec)
    out = {}
    for i, recs in parts.items():
        recs.sort(key=lambda r: r["start"])
        assert sum(r["n"] for r in recs) == man["numels"][i]
        for r in recs:
            assert r["start"] % B == 0
        out[i] = {k: torch.cat([r[k] for r in recs]) for k in
                  ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min")}
    return man, out


def _big_worker(rank, world, port, sizes, src, dst, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _use_oracle()
        from mdq_b200.zero1 import ZeroMDQAdamW

        torch.set_num_threads(2)
        g = torch.Generator().manual_seed(5)
        params = [torch.nn.Parameter(torch.randn(n, generator=g) * 0.02) for n in sizes]
        opt = ZeroMDQAdamW(params, lr=1e-3, weight_decay=0.01, block_size=256, fixed_bits=4)
        if src is None:
            opt.zero_grad()
            gg = torch.Generator().manual_seed(100 + rank)
            for p in params:
                p.grad.copy_(torch.randn(p.numel(), generator=gg).view_as(p) * 1e-3)
            opt.step()
        else:
            opt.load_sharded(src)
        opt.save_sharded(dst)
        q.put(rank)
    finally:
        dist.destroy_process_group()


def _spawn_big(world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_big_worker, args=(r, world, port) + args + (q,))
             for r in range(world)]
    for p in procs:
        p.start()
    for _ in range(world):
        q.get(timeout=600)
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0


def test_sharded_checkpoint_1e8_elements_2_to_3_ranks(tmp_path):
    """10^8 elements: one step at 2 ranks, save_sharded; load_sharded at 3
    ranks and save again.  Both checkpoints hold the same full codes and
    scales, every piece block-aligned; no rank ever gathers the state."""
    sizes = [60_000_001, 39_999_743, 256]
    a, b = str(tmp_path / "w2"), str(tmp_path / "w3")
    _spawn_big(2, sizes, None, a)
    _spawn_big(3, sizes, a, b)
    man_a, full_a = _reconstruct(a)
    man_b, full_b = _reconstruct(b)
    assert (man_a["world"], man_b["world"]) == (2, 3)
    assert man_a["params"] == man_b["params"]
    for i in range(len(sizes)):
        for k, t in full_a[i].items():
            assert torch.equal(t.view(torch.uint8), full_b[i][k].view(torch.uint8)), (i, k)
    # the state is not trivial: the step moved the scales off their initial values
    assert not torch.equal(full_a[0]["v_min"], torch.full_like(full_a[0]["v_min"], -20.0))


def _bf16_resume_worker(rank, world, port, sizes, phase, payload, q):
    """bf16 parameters: phase "save" runs steps 1-3 and returns the
    consolidated state (with fp32 masters); phase "resume" loads it at this
    world size and runs steps 4-6.  Gradients are every rank's average."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _use_oracle()
        from mdq_b200.zero1 import ZeroMDQAdamW

        torch.set_num_threads(1)
        params = _params(sizes)
        opt = ZeroMDQAdamW(params, lr=1e-3, weight_decay=0.01, block_size=256, fixed_bits=(8, 4),
                           param_dtype=torch.bfloat16, bucket_elems=3000)
        steps = range(1, 4)
        if phase == "resume":
            opt.load_consolidated_state_dict(_torch_tree(payload))
            steps = range(4, 7)
        for t in steps:
            opt.zero_grad()
            avg = [sum(gs) / 2 for gs in zip(*[_bf16_grads(r, t, sizes) for r in range(2)])]
            for p, g in zip(params, avg):
                p.grad.copy_(g.to(torch.bfloat16))
            opt.step()
        sd = opt.consolidated_state_dict(dst=0)
        if rank == 0:
            q.put((_np_tree(sd), [p.detach().float().numpy().copy() for p in params]))
    finally:
        dist.destroy_process_group()


def test_bf16_consolidated_resume_restores_masters():
    """The consolidated state of a bf16-parameter run carries the fp32
    masters: resumed at another world size, 3 + 3 steps equal 6 unsharded
    fp32 steps bit for bit (masters), and the parameters are their bf16."""
    sizes = SIZES
    _use_oracle()
    from mdq_b200.optim import MDQAdamWSimpleFusedIO

    torch.set_num_threads(1)
    ref = _params(sizes)
    ref_opt = MDQAdamWSimpleFusedIO(ref, lr=1e-3, weight_decay=0.01, block_size=256,
                                    fixed_bits=(8, 4))
    for t in range(1, 7):
        avg = [sum(gs) / 2 for gs in zip(*[_bf16_grads(r, t, sizes) for r in range(2)])]
        for p, g in zip(ref, avg):
            p.grad_dtype = torch.bfloat16
            p.grad = g.to(torch.bfloat16)
        ref_opt.step()

    def spawn(world, phase, payload):
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_bf16_resume_worker,
                             args=(r, world, port, sizes, phase, payload, q)) for r in range(world)]
        for p in procs:
            p.start()
        out = q.get(timeout=300)
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        return out

    saved, _ = spawn(2, "save", None)
    sd, model = spawn(3, "resume", saved)
    sd = _torch_tree(sd)
    for i, p in enumerate(ref):
        want = p.detach()
        assert torch.equal(sd["state"][i]["master"].view(torch.int32), want.view(torch.int32)), i
        np.testing.assert_array_equal(model[i], want.to(torch.bfloat16).float().numpy())
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            np.testing.assert_array_equal(ref_opt.state[p][k].numpy().view(np.uint8),
                                          sd["state"][i][k].numpy().view(np.uint8))
