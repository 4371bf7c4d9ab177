"""The multi-GPU D-slab TV path over NCCL (2 ranks, one GPU each) against the
single-GPU result on the whole volume. Skipped on a box with fewer than 2 GPUs
(the host logic is covered on CPU ranks in test_sharded_cpu.py)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPE = (2, 46, 40, 132)  # D split 23 + 23 across 2 ranks


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _volume():
    gen = torch.Generator().manual_seed(31)
    return torch.rand(SHAPE, generator=gen)


def _worker(rank, world, port, queue):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from quantem.cuda import sharded

        vol = _volume()
        B, D, H, W = SHAPE
        lo, hi = sharded.slab_bounds(D, rank, world)
        slab = torch.zeros((B, hi - lo + 2, H, W), device="cuda")
        slab[:, 1 : hi - lo + 1] = vol[:, lo:hi].cuda()
        out = {}
        for variant, g, eps in ((sharded.SQ, [1.5], 0.0), (sharded.ISO, [0.75], 1e-6), (sharded.L1, [0.3, 1.1, 0.6], 0.0)):
            loss, grad = sharded.tv_loss_slab_fwd_grad(variant, slab, torch.tensor(g, device="cuda"), D, eps)
            out[variant] = (loss.cpu().numpy(), grad[:, 1 : hi - lo + 1].cpu().numpy())
        queue.put((rank, lo, hi, out))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dslab_over_nccl_matches_single_gpu():
    from quantem.cuda.core import tv_loss_iso_3d_fwd_grad, tv_loss_l1_3d_fwd_grad, tv_loss_sq_3d_fwd_grad

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    v = _volume().cuda()
    whole = {
        0: tv_loss_sq_3d_fwd_grad(v, 1.5),
        1: tv_loss_iso_3d_fwd_grad(v, 0.75, eps=1e-6),
        2: tv_loss_l1_3d_fwd_grad(v, (0.3, 1.1, 0.6)),
    }
    for variant, (loss, grad) in whole.items():
        loss, grad = loss.cpu().numpy(), grad.cpu().numpy()
        for rank, lo, hi, out in res:
            r_loss, r_grad = out[variant]
            np.testing.assert_allclose(np.atleast_1d(r_loss), np.atleast_1d(loss), rtol=1e-5)
            np.testing.assert_allclose(r_grad, grad[:, lo:hi], rtol=1e-5, atol=1e-6 * np.abs(grad).max())
