"""Host logic of the multi-GPU forms on CPU ranks (gloo, world_size 2 and 3):
D-slab halo exchange, ownership flags, the global isotropic normalisation and
the rank-ordered loss sum for TV; the plane/rotation gradient all-reduce for
point-sharded K-Planes. The per-rank device kernel is replaced by the CPU
oracle, so every rank's result can be compared with the oracle on the whole
problem."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle

SQ, ISO, L1 = 0, 1, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_slab_kernel(variant, flags, slab, g, acc, grad, d_lo, d_hi, has_prev, has_next, eps, scale):
    """The slab semantics of tv_loss_3d_slab_cuda computed with the oracle on
    the planes this rank holds (its owned planes plus the halos it received)."""
    x = slab.numpy()
    lo = d_lo - (1 if has_prev else 0)
    hi = d_hi + (1 if has_next else 0)
    window = np.ascontiguousarray(x[:, lo:hi])
    gv = g.numpy().astype(np.float64) * scale
    if variant == SQ:
        gw = oracle.tv_sq_grad(window, float(gv[0]))
    elif variant == ISO:
        gw = oracle.tv_iso_grad(window, float(gv[0]), eps)
    else:
        gw = oracle.tv_l1_grad(window, gv.astype(np.float32))
    off = d_lo - lo
    grad[:, d_lo:d_hi] = torch.from_numpy(gw[:, off : off + (d_hi - d_lo)])
    fwd = np.ascontiguousarray(x[:, d_lo:hi])  # owned planes + the next halo
    nxt = np.ascontiguousarray(x[:, d_hi : d_hi + 1])
    if variant == SQ:
        loss = np.array([oracle.tv_sq_loss(fwd) - (oracle.tv_sq_loss(nxt) if has_next else 0.0)])
    elif variant == L1:
        loss = oracle.tv_l1_loss(fwd) - (oracle.tv_l1_loss(nxt) if has_next else 0.0)
    else:
        loss = np.array([oracle.tv_iso_sum(fwd, eps)])
    acc.copy_(torch.from_numpy((loss * scale).astype(np.float32)))


def _tv_worker(rank, world, port, shape, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from quantem.cuda import sharded

        B, D, H, W = shape
        gen = torch.Generator().manual_seed(5)
        vol = torch.rand(shape, generator=gen)
        lo, hi = sharded.slab_bounds(D, rank, world)
        results = {}
        for variant, g, eps in ((SQ, torch.tensor([1.5]), 0.0), (ISO, torch.tensor([0.75]), 1e-6),
                                (L1, torch.tensor([0.3, 1.1, 0.6]), 0.0)):
            slab = torch.zeros((B, hi - lo + 2, H, W))
            slab[:, 1 : hi - lo + 1] = vol[:, lo:hi]  # halos arrive through exchange_halos
            loss, grad = sharded.tv_loss_slab_fwd_grad(variant, slab, g, D, eps, slab_kernel=oracle_slab_kernel)
            results[variant] = (loss.numpy().copy(), grad[:, 1 : hi - lo + 1].numpy().copy())
        queue.put((rank, lo, hi, results))
    finally:
        dist.destroy_process_group()


def _run(worker, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out, key=lambda t: t[0])


# uneven slabs (11 planes over 2 and 3 ranks), and ranks that own a single
# plane, whose two halos both come from neighbours (5 planes over 4 ranks)
@pytest.mark.parametrize("world,shape", [(2, (2, 11, 9, 12)), (3, (2, 11, 9, 12)), (4, (1, 5, 6, 8))])
def test_tv_dslab_matches_whole_volume(world, shape):
    out = _run(_tv_worker, world, shape)
    gen = torch.Generator().manual_seed(5)
    x = torch.rand(shape, generator=gen).numpy()
    B, D, H, W = shape
    n = B * (D - 1) * (H - 1) * (W - 1)
    # losses are g-independent (raw sums for SQ and L1, the mean for ISO);
    # gradients carry the upstream factors
    want = {
        SQ: (np.array([oracle.tv_sq_loss(x)]), oracle.tv_sq_grad(x, 1.5)),
        ISO: (np.array([oracle.tv_iso_sum(x, 1e-6) / n]), oracle.tv_iso_grad(x, 0.75 / n, 1e-6)),
        L1: (oracle.tv_l1_loss(x), oracle.tv_l1_grad(x, [0.3, 1.1, 0.6])),
    }
    losses = {v: [] for v in want}
    for rank, lo, hi, res in out:
        for v, (loss, grad) in res.items():
            losses[v].append(np.atleast_1d(loss))
            np.testing.assert_allclose(grad, want[v][1][:, lo:hi], rtol=1e-5, atol=1e-7)
    for v, ls in losses.items():
        for loss in ls:  # bitwise identical on every rank
            np.testing.assert_array_equal(loss, ls[0])
        np.testing.assert_allclose(ls[0], want[v][0], rtol=1e-5)


def test_rotation_buckets_partition():
    from quantem.cuda.sharded import _rotation_buckets

    for T in (1, 2, 3, 4, 8, 13):
        for k in (0, 1, 2, 3, 4, 16):
            ranges = _rotation_buckets(T, k)
            assert ranges[0][0] == 0 and ranges[-1][1] == T
            assert all(a[1] == b[0] and a[1] > a[0] for a, b in zip(ranges, ranges[1:]))
            assert len(ranges) == max(1, min(k, T))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_slab_bounds_partition():
    from quantem.cuda import sharded

    for D in (1, 7, 256, 1000):
        for world in (1, 2, 3, 8):
            spans = [sharded.slab_bounds(D, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == D
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


def oracle_fwd_bwd(pts, rot, plane, gout):
    out = torch.from_numpy(oracle.kplanes_fwd(pts.numpy(), rot.numpy(), plane.numpy()))
    gp, gr, gg = oracle.kplanes_bwd(pts.numpy(), rot.numpy(), plane.numpy(), gout.numpy())
    return out, torch.from_numpy(gp), torch.from_numpy(gr), torch.from_numpy(gg)


def _kp_worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from quantem.cuda import sharded

        N, T, C, H, W = 300, 2, 8, 9, 11
        gen = torch.Generator().manual_seed(6)
        pts = torch.empty((N, 3)).uniform_(-1.05, 1.05, generator=gen)
        rot = torch.empty((T, 3, 3)).uniform_(-1, 1, generator=gen)
        plane = torch.empty((3 * T, C, H, W)).uniform_(0.1, 0.5, generator=gen)
        up = torch.randn((N, T * C), generator=gen)
        lo, hi = sharded.slab_bounds(N, rank, world)
        out, gp, gr, gg, work = sharded.kplanes_fwd_bwd_sharded(
            pts[lo:hi], rot, plane, up[lo:hi], async_op=True, fwd_bwd=oracle_fwd_bwd
        )
        work.wait()
        queue.put((rank, lo, hi, out.numpy(), gp.numpy(), gr.numpy(), gg.numpy()))
    finally:
        dist.destroy_process_group()


def test_kplanes_point_sharding_reduces_plane_gradients():
    world = 2
    out = _run(_kp_worker, world)
    N, T, C, H, W = 300, 2, 8, 9, 11
    gen = torch.Generator().manual_seed(6)
    pts = torch.empty((N, 3)).uniform_(-1.05, 1.05, generator=gen)
    rot = torch.empty((T, 3, 3)).uniform_(-1, 1, generator=gen)
    plane = torch.empty((3 * T, C, H, W)).uniform_(0.1, 0.5, generator=gen)
    up = torch.randn((N, T * C), generator=gen)
    o_out, o_gp, o_gr, o_gg = oracle_fwd_bwd(pts, rot, plane, up)
    for rank, lo, hi, o, gp, gr, gg in out:
        np.testing.assert_allclose(o, o_out[lo:hi].numpy(), rtol=1e-6)
        np.testing.assert_allclose(gp, o_gp[lo:hi].numpy(), rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(gr, o_gr.numpy(), rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(gg, o_gg.numpy(), rtol=1e-5, atol=1e-7)


# ── failures on the host: a rank that stops, a neighbour with another shape ──


def _dead_rank_worker(rank, world, port, queue):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from quantem.cuda import sharded

    if rank == world - 1:
        # this rank stops before the step: it never sends its halo
        queue.put((rank, "left"))
        queue.close()
        queue.join_thread()
        os._exit(0)
    slab = torch.rand((1, 6, 4, 8))
    try:
        sharded.tv_loss_slab_fwd_grad(SQ, slab, torch.tensor([1.0]), 4 * world, slab_kernel=oracle_slab_kernel)
        queue.put((rank, "no error"))
    except Exception as e:  # the collective gives up after the group's timeout
        queue.put((rank, f"detected: {type(e).__name__}"))
    queue.close()
    queue.join_thread()
    os._exit(0)


def test_a_rank_that_stops_is_detected_by_its_neighbours():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = dict(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert out[world - 1] == "left"
    assert out[0].startswith("detected"), out[0]


def _shape_mismatch_worker(rank, world, port, queue):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    from quantem.cuda import sharded

    # rank 1's planes are wider than rank 0's: the halo exchange must fail
    slab = torch.rand((1, 6, 4, 8 if rank == 0 else 12))
    try:
        sharded.exchange_halos(slab)
        queue.put((rank, "no error"))
    except Exception as e:
        queue.put((rank, f"detected: {type(e).__name__}"))
    queue.close()
    queue.join_thread()
    os._exit(0)


def test_a_neighbour_with_another_plane_shape_is_rejected():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shape_mismatch_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = dict(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert all(v == "detected: ValueError" for v in out.values()), out


def test_peer_objects_reject_ranks_that_disagree():
    from quantem.cuda.sharded import _same_on_every_rank

    _same_on_every_rank([(2, 64, 8, 8)] * 4, "shape")
    with pytest.raises(ValueError, match="rank 2"):
        _same_on_every_rank([(2, 64, 8, 8), (2, 64, 8, 8), (2, 64, 8, 9)], "PeerSlab shape")


def test_peer_mappings_are_closed_when_construction_fails(monkeypatch):
    from quantem.cuda import _core, sharded

    closed = []
    monkeypatch.setattr(_core, "ipc_close", lambda ptr: closed.append(ptr))
    mapped = [11, 22]
    with pytest.raises(KeyError):
        with sharded._unmap_on_error(mapped):
            mapped.append(33)
            raise KeyError("the third handle would not open")
    assert closed == [11, 22, 33] and mapped == []
    # nothing is closed when construction succeeds
    ok = [44]
    with sharded._unmap_on_error(ok):
        pass
    assert ok == [44] and closed == [11, 22, 33]
