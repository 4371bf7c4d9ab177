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


# ── D-slabs over peer memory (CUDA IPC, stores over NVLink) ──────────────────

# D split 23 + 22 (slabs of different depth) on the TMA path, and an odd width
# on the generic path (which exchanges with a separate kernel)
PEER_SHAPES = [(2, 45, 40, 132), (1, 9, 7, 10)]
PEER_STEPS = 3
PEER_CASES = ((0, [1.5], 0.0), (1, [0.75], 1e-6), (2, [0.3, 1.1, 0.6], 0.0))  # SQ, ISO, L1


def _peer_volume(shape, step: int):
    gen = torch.Generator().manual_seed(100 + step)
    return torch.rand(shape, generator=gen)


def _peer_worker(rank, world, port, queue, shape):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ps = None
    try:
        from quantem.cuda import _core, sharded

        B, D, H, W = shape
        ps = sharded.PeerSlab(B, D, H, W, timeout_s=20.0)
        lo, hi = ps.d_lo, ps.d_hi
        out = []
        for step in range(PEER_STEPS):
            # the volume changes between steps, so stale halos would show
            ps.owned.copy_(_peer_volume(shape, step)[:, lo:hi].cuda())
            per = {}
            if step == 2:
                # all three losses with one cross-rank finalize
                res = ps.fwd_grad_many([(v, torch.tensor(g), eps) for v, g, eps in PEER_CASES])
                for (variant, _, _), (loss, grad) in zip(PEER_CASES, res):
                    per[variant] = (loss.cpu().numpy(), grad[:, 1:-1].cpu().numpy())
            for variant, g, eps in PEER_CASES if step < 2 else ():
                if step == 1:
                    # the exchange as its own kernel, then the sweep without one
                    ps.exchange_halos()
                    loss, grad = ps.fwd_grad(variant, torch.tensor(g), eps, exchange=False)
                else:
                    # the exchange inside the sweep kernel
                    loss, grad = ps.fwd_grad(variant, torch.tensor(g), eps)
                per[variant] = (loss.cpu().numpy(), grad[:, 1:-1].cpu().numpy())
            out.append(per)
        fault = _core.device_fault_word(rank)
        queue.put((rank, lo, hi, out, fault))
        ps.close()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


# 2 ranks (both at an end of the volume), and 4 and 8 ranks (interior ranks
# with a neighbour on each side) where the box has them
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("shape", PEER_SHAPES)
def test_peer_slab_matches_single_gpu_over_steps(shape, world):
    from quantem.cuda.core import tv_loss_iso_3d_fwd_grad, tv_loss_l1_3d_fwd_grad, tv_loss_sq_3d_fwd_grad

    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q, shape)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, _, _, _, fault in res:
        assert fault == 0, f"rank {rank} gave up waiting (fault word {fault:#x})"
    fns = {0: tv_loss_sq_3d_fwd_grad, 1: tv_loss_iso_3d_fwd_grad, 2: tv_loss_l1_3d_fwd_grad}
    for step in range(PEER_STEPS):
        v = _peer_volume(shape, step).cuda()
        for variant, g, eps in PEER_CASES:
            kw = {"eps": eps} if variant == 1 else {}
            loss, grad = fns[variant](v, g[0] if len(g) == 1 else tuple(g), **kw)
            loss, grad = np.atleast_1d(loss.cpu().numpy()), grad.cpu().numpy()
            losses = []
            for rank, lo, hi, out, _ in res:
                r_loss, r_grad = out[step][variant]
                losses.append(np.atleast_1d(r_loss))
                np.testing.assert_allclose(np.atleast_1d(r_loss), loss, rtol=1e-5)
                np.testing.assert_allclose(r_grad, grad[:, lo:hi], rtol=1e-5, atol=1e-6 * np.abs(grad).max())
            # the rank-ordered sum gives every rank the same bits
            assert all(np.array_equal(losses[0], x) for x in losses[1:])


# ── K-Planes over points, per-rotation gradient all_reduce ───────────────────

KP_CFG = (6000, 4, 32, 40, 36)  # N, T, C, H, W


def _kp_inputs():
    N, T, C, H, W = KP_CFG
    gen = torch.Generator().manual_seed(77)
    pts = torch.empty((N, 3)).uniform_(-1.1, 1.1, generator=gen)
    rot = torch.empty((T, 3, 3)).uniform_(-1.0, 1.0, generator=gen)
    plane = torch.empty((3 * T, C, H, W)).uniform_(0.1, 0.5, generator=gen)
    up = torch.randn((N, T * C), generator=gen)
    return pts, rot, plane, up


def _kp_worker(rank, world, port, queue):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from quantem.cuda import sharded

        pts, rot, plane, up = _kp_inputs()
        lo, hi = sharded.slab_bounds(pts.shape[0], rank, world)
        p, r, g, u = pts[lo:hi].cuda(), rot.cuda(), plane.cuda(), up[lo:hi].cuda()
        out, g_pts, g_rot, g_plane, work = sharded.kplanes_fwd_bwd_sharded(p, r, g, u, async_op=True)
        work.wait()
        # the same step with the gradients summed over peer memory, twice
        reducer = sharded.kplanes_gradient_reducer(g, r)
        for _ in range(2):
            _, pg_pts, pg_rot, pg_plane, pwork = sharded.kplanes_fwd_bwd_sharded(p, r, g, u, reducer=reducer,
                                                                                buckets=1)
        assert pwork is None
        # and with the backward in three rotation buckets, each bucket's sum
        # on the reducer's second stream beside the next bucket's backward
        for _ in range(2):
            _, bg_pts, bg_rot, bg_plane, _ = sharded.kplanes_fwd_bwd_sharded(p, r, g, u, reducer=reducer,
                                                                             buckets=3, reduce_ctas=8)
        torch.cuda.synchronize()
        from quantem.cuda import _core

        fault = _core.peer_allreduce_fault_word(rank)
        reducer.close()
        queue.put((rank, lo, hi, out.cpu(), g_pts.cpu(), g_rot.cpu(), g_plane.cpu(),
                   pg_pts.cpu(), pg_rot.cpu(), pg_plane.cpu(), fault,
                   bg_pts.cpu(), bg_rot.cpu(), bg_plane.cpu()))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kplanes_point_sharding_matches_single_gpu():
    import quantem.cuda.core.ml  # noqa: F401  (registers the K-Planes ops used below)

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_kp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    pts, rot, plane, up = (t.cuda() for t in _kp_inputs())
    out = torch.ops.quantem_cuda.kplanes_tilted_fuse(pts, rot, plane).cpu()
    ref_pts, ref_rot, ref_plane = (t.cpu() for t in torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(pts, rot, plane, up))
    for rank, lo, hi, r_out, r_pts, r_rot, r_plane, p_pts, p_rot, p_plane, fault, b_pts, b_rot, b_plane in res:
        assert fault == 0
        assert torch.equal(r_out, out[lo:hi])
        for gp, gr, gg in ((r_pts, r_rot, r_plane), (p_pts, p_rot, p_plane), (b_pts, b_rot, b_plane)):
            torch.testing.assert_close(gp, ref_pts[lo:hi], rtol=1e-4, atol=1e-5 * ref_pts.abs().max().item())
            torch.testing.assert_close(gr, ref_rot, rtol=1e-4, atol=1e-4 * ref_rot.abs().max().item())
            torch.testing.assert_close(gg, ref_plane, rtol=1e-4, atol=1e-5 * ref_plane.abs().max().item())
    # both reductions give every rank the same gradients
    assert torch.equal(res[0][5], res[1][5]) and torch.equal(res[0][6], res[1][6])
    assert torch.equal(res[0][8], res[1][8]) and torch.equal(res[0][9], res[1][9])
    assert torch.equal(res[0][12], res[1][12]) and torch.equal(res[0][13], res[1][13])



# ── the peer-memory all-reduce on its own ────────────────────────────────────


# Sizes: fewer elements than 4 x ranks (tail only), one float4 per rank plus
# a tail, and a large size that is not a multiple of 4 x ranks.
ALLREDUCE_SIZES = (3, 37, 1_000_003)
# (offset, count, max_ctas) of ranged sums: inside one float4, across a
# boundary, an unaligned start with a long body and tail, an empty range
RANGES = ((1, 2, 1), (2, 9, 0), (5, 999_990, 3), (36, 0, 1))


def _allreduce_worker(rank, world, port, queue):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from quantem.cuda import _core, sharded

        outs = []
        for n in ALLREDUCE_SIZES:
            red = sharded.PeerAllReduce(n, timeout_s=20.0)
            for call in range(3):
                gen = torch.Generator().manual_seed(1000 * call + rank)
                red.buffer.copy_(torch.randn(n, generator=gen).cuda())
                outs.append(red.all_reduce().cpu().clone())
            # ranges with unaligned ends, few CTAs: only the range is summed
            for lo, cnt, ctas in RANGES:
                if lo + cnt > n:
                    continue
                gen = torch.Generator().manual_seed(7000 + rank)
                red.buffer.copy_(torch.randn(n, generator=gen).cuda())
                red.all_reduce(lo, cnt, ctas)
                outs.append(red.buffer.cpu().clone())
            torch.cuda.synchronize()
            red.close()
        queue.put((rank, outs, _core.peer_allreduce_fault_word(rank)))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_allreduce_is_the_rank_ordered_sum(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_allreduce_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    k = 0
    for n in ALLREDUCE_SIZES:
        for call in range(3):
            parts = [torch.randn(n, generator=torch.Generator().manual_seed(1000 * call + r)) for r in range(world)]
            expect = parts[0].clone()
            for x in parts[1:]:
                expect += x  # fp32, rank order: what the kernel computes
            for rank, outs, fault in res:
                assert fault == 0
                assert torch.equal(outs[k], expect), (rank, n, call)
            k += 1
        for lo, cnt, _ in RANGES:
            if lo + cnt > n:
                continue
            parts = [torch.randn(n, generator=torch.Generator().manual_seed(7000 + r)) for r in range(world)]
            total = parts[0].clone()
            for x in parts[1:]:
                total += x
            for rank, outs, fault in res:
                expect = parts[rank].clone()
                expect[lo : lo + cnt] = total[lo : lo + cnt]
                assert torch.equal(outs[k], expect), (rank, n, lo, cnt)
            k += 1
