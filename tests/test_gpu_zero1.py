"""ZeRO-1 on real GPUs with NCCL (needs >= 2 devices; skipped otherwise):
reduce-scatter / fused step / all-gather equals the unsharded optimizer on one
GPU with the averaged gradients, bit for bit (fixed bit widths, exact p), also
with bucketed reduce-scatters launched during backward."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SIZES = [1000, 3, (1 << 20) + 17, 256, 777, 2048, 1, 65536 * 3 + 5]


def _grads(rank, step):
    g = torch.Generator().manual_seed(1000 * step + rank)
    return [torch.round(torch.randn(n, generator=g) * 1024 * 2.0 ** (i % 3)) / 2 ** 20
            for i, n in enumerate(SIZES)]


def _params(device):
    g = torch.Generator().manual_seed(0)
    return [torch.nn.Parameter((torch.randn(n, generator=g) * 0.02).to(device)) for n in SIZES]


KW = dict(lr=1e-3, weight_decay=0.01, block_size=256, p_mode="exact")


def _worker(rank, world, port, steps, bits, overlap, q, gather="nccl"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        from mdq_b200.zero1 import ZeroMDQAdamW

        params = _params(torch.device("cuda", rank))
        extra = dict(bucket_elems=300_000, overlap_grad_reduce=True) if overlap else {}
        opt = ZeroMDQAdamW([{"params": params[:4]}, {"params": params[4:], "weight_decay": 0.0}],
                           fixed_bits=bits, param_gather=gather.split("+")[0],
                           grad_reduce="peer" if gather.endswith("+grad") else "nccl",
                           **KW, **extra)
        for t in range(1, steps + 1):
            opt.zero_grad()
            if overlap:
                # Gradients from backward (loss = sum_i <p_i, c_i>): the bucket
                # reduce-scatters start from the hooks, during backward.
                coef = [c.to(params[0].device) for c in _grads(rank, t)]
                sum((p * c).sum() for p, c in zip(params, coef)).backward()
            else:
                for p, g in zip(params, _grads(rank, t)):
                    p.grad.copy_(g)
            opt.step()
        torch.cuda.synchronize()
        sd = opt.consolidated_state_dict()
        if rank == 0:
            q.put(([p.detach().cpu().numpy() for p in params],
                   {i: {k: (v.numpy() if torch.is_tensor(v) else v) for k, v in st.items()}
                    for i, st in sd["state"].items()}))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bits,overlap,gather", [(4, False, "nccl"), ((8, 4), False, "nccl"),
                                                 (8, False, "nccl"), ((8, 4), True, "nccl"),
                                                 ((8, 4), False, "peer"), (4, True, "peer"),
                                                 ((8, 4), False, "peer+grad"), (8, False, "peer+grad")])
def test_zero1_nccl_equals_unsharded(cuda_device, bits, overlap, gather):
    """gather "peer": the step kernel itself stores the updated parameters
    into every rank's copy (symmetric memory) instead of an NCCL all-gather;
    "peer+grad": it also sums every rank's gradients instead of an NCCL
    reduce-scatter."""
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    from mdq_b200.optim import MDQAdamWSimpleFusedIO

    steps = 4
    params = _params(cuda_device)
    opt = MDQAdamWSimpleFusedIO([{"params": params[:4]}, {"params": params[4:], "weight_decay": 0.0}],
                                fixed_bits=bits, **KW)
    for t in range(1, steps + 1):
        per = [_grads(r, t) for r in range(world)]
        for i, p in enumerate(params):
            p.grad = (sum(pr[i] for pr in per) / world).to(cuda_device)
        opt.step()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, steps, bits, overlap, q, gather))
             for r in range(world)]
    for p in procs:
        p.start()
    got_params, state = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for i, (a, b) in enumerate(zip(params, got_params)):
        np.testing.assert_array_equal(a.detach().cpu().numpy().view(np.int32), b.view(np.int32),
                                      err_msg=f"param {i}")
        rs = opt.state[a]
        for k in ("exp_avg", "exp_avg_sq", "scale_m", "scale_v", "v_min"):
            np.testing.assert_array_equal(rs[k].cpu().numpy().view(np.uint8),
                                          state[i][k].view(np.uint8), err_msg=f"param {i} {k}")
