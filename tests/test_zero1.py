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


def test_layout_is_block_aligned_and_covers_every_element():
    for world in (1, 2, 3, 8):
        lay = ShardLayout(SIZES, 256, world)
        assert lay.total % (world * 256) == 0
        seen = {i: 0 for i in range(len(SIZES))}
        for r in range(world):
            for pc in lay.pieces(r):
                assert pc.flat_off % 256 == 0 and pc.start % 256 == 0
                assert r * lay.shard <= pc.flat_off and pc.flat_off + pc.n <= (r + 1) * lay.shard
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
