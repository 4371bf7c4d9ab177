"""Multi-GPU forms of the hot path: one process per GPU, torch.distributed
(NCCL over NVLink on GPUs; any backend for the host logic).

Neither exists in the reference (quantem-cuda is single-GPU); both follow the
natural sharding of the work:

* TV over D-slabs. Each rank owns a contiguous range of planes of every batch
  slice, stored with one halo plane on each side: ``slab [B, D_local + 2, H, W]``
  (planes 1..D_local owned). :func:`exchange_halos` fills the halo planes from
  the neighbouring ranks; the single-sweep kernel then computes the loss terms
  anchored at owned planes and the gradient of owned planes
  (``tv_loss_3d_slab_cuda``). The per-rank sums are all-gathered and added in
  rank order, so the total is deterministic and identical on every rank.

* K-Planes over points. Each rank evaluates its own points against the
  replicated planes and rotations; point gradients stay local, and the plane
  and rotation gradients are summed with all_reduce.

The per-rank compute defaults to the CUDA kernels. ``slab_kernel`` exists so
that the host logic (halo exchange, ownership flags, reductions) can be tested
on CPU ranks with the CPU oracle in place of the device kernel.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist
from torch import Tensor

SQ, ISO, L1 = 0, 1, 2
_N_ACC = {SQ: 1, ISO: 1, L1: 3}
_LOSS, _GRAD, _OVERWRITE = 1, 2, 4


def _rank_world(group) -> tuple[int, int]:
    return dist.get_rank(group), dist.get_world_size(group)


def _peer(group, r: int) -> int:
    return r if group is None else dist.get_global_rank(group, r)


def slab_bounds(global_d: int, rank: int, world: int) -> tuple[int, int]:
    """Owned global planes [lo, hi) of `rank` for a D-split over `world` ranks
    (contiguous, sizes differing by at most one)."""
    base, extra = divmod(global_d, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def exchange_halos(slab: Tensor, group=None) -> None:
    """Fills the halo planes 0 and -1 of ``slab [B, D_local + 2, H, W]`` with
    the neighbouring ranks' boundary planes (rank r-1's last owned plane and
    rank r+1's first). Ranks at the ends of the global volume leave that halo
    as it is (the kernel is told it is not a neighbour)."""
    rank, world = _rank_world(group)
    if world == 1:
        return
    d_local = slab.shape[1] - 2
    send_lo = slab[:, 1].contiguous()
    send_hi = slab[:, d_local].contiguous()
    recv_lo = torch.empty_like(send_lo)
    recv_hi = torch.empty_like(send_hi)
    ops = []
    if rank > 0:
        ops.append(dist.P2POp(dist.isend, send_lo, _peer(group, rank - 1), group))
        ops.append(dist.P2POp(dist.irecv, recv_lo, _peer(group, rank - 1), group))
    if rank < world - 1:
        ops.append(dist.P2POp(dist.isend, send_hi, _peer(group, rank + 1), group))
        ops.append(dist.P2POp(dist.irecv, recv_hi, _peer(group, rank + 1), group))
    for req in dist.batch_isend_irecv(ops):
        req.wait()
    if rank > 0:
        slab[:, 0].copy_(recv_lo)
    if rank < world - 1:
        slab[:, d_local + 1].copy_(recv_hi)


def _cuda_slab_kernel(variant, flags, vol, g, acc, grad, d_lo, d_hi, has_prev, has_next, eps, scale):
    from quantem.cuda import _core
    from quantem.cuda._common import _workspace

    b, dp, h, w = vol.shape
    ws = _workspace(vol.device)
    with torch.cuda.device(vol.device):
        _core.tv_loss_3d_slab_cuda(
            variant, flags, vol.data_ptr(), g.data_ptr(), acc.data_ptr(),
            grad.data_ptr(), b, dp, h, w, d_lo, d_hi, int(has_prev), int(has_next),
            float(eps), float(scale), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream(vol.device).cuda_stream,
        )


def reduce_in_rank_order(local: Tensor, group=None) -> Tensor:
    """Sum of `local` over ranks, added in rank order in fp64 (deterministic,
    bitwise identical on every rank)."""
    _, world = _rank_world(group)
    if world == 1:
        return local
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    total = torch.zeros(local.shape, dtype=torch.float64, device=local.device)
    for p in parts:
        total += p.double()
    return total.to(local.dtype)


def tv_loss_slab_fwd_grad(
    variant: int,
    slab: Tensor,
    grad_out: Tensor,
    global_d: int,
    eps: float = 1e-8,
    group=None,
    exchange: bool = True,
    slab_kernel: Callable | None = None,
) -> tuple[Tensor, Tensor]:
    """Loss and gradient of one TV variant over a D-sharded volume.

    Args:
        variant:  SQ, ISO or L1.
        slab:     ``[B, D_local + 2, H, W]`` fp32, owned planes 1..D_local,
                  halos at 0 and D_local + 1 (filled here when ``exchange``).
        grad_out: upstream gradient, shape (1,) (SQ, ISO) or (3,) (L1).
        global_d: D of the whole volume (the isotropic mean divides by the
                  global corner count).

    Returns:
        ``(loss, grad)``: the global loss (identical on every rank; the mean
        for ISO, raw sums for SQ and L1) and ``grad [B, D_local + 2, H, W]``
        whose owned planes hold this rank's part of the gradient.
    """
    rank, world = _rank_world(group)
    if exchange:
        exchange_halos(slab, group)
    b, dp, h, w = slab.shape
    d_local = dp - 2
    scale = 1.0
    if variant == ISO:
        scale = 1.0 / max(1, b * (global_d - 1) * (h - 1) * (w - 1))
    acc = torch.empty(_N_ACC[variant], dtype=torch.float32, device=slab.device)
    grad = torch.empty_like(slab)
    kern = slab_kernel or _cuda_slab_kernel
    kern(variant, _LOSS | _GRAD | _OVERWRITE, slab, grad_out, acc, grad, 1, d_local + 1,
         rank > 0, rank < world - 1, eps, scale)
    loss = reduce_in_rank_order(acc, group)
    return (loss.squeeze(0) if variant != L1 else loss), grad


def kplanes_fwd_bwd_sharded(
    pts_local: Tensor,
    rotations: Tensor,
    plane: Tensor,
    grad_out_local: Tensor,
    group=None,
    async_op: bool = False,
    fwd_bwd: Callable | None = None,
):
    """Forward and backward of one K-Planes level over point-sharded ranks.

    Returns ``(out_local, grad_pts_local, grad_rotations, grad_plane, work)``:
    the plane and rotation gradients are summed over ranks with all_reduce
    (``work`` is the pending collective when ``async_op``, so that the next
    level's compute overlaps it; call ``work.wait()`` before reading them).
    ``fwd_bwd(pts, rotations, plane, grad_out) -> (out, g_pts, g_rot, g_plane)``
    replaces the CUDA ops (host-logic tests on CPU ranks).
    """
    if fwd_bwd is None:
        from quantem.cuda.core.ml._ops import _kplanes_tilted_fuse, _kplanes_tilted_fuse_bwd

        out = _kplanes_tilted_fuse(pts_local, rotations, plane)
        g_pts, g_rot, g_plane = _kplanes_tilted_fuse_bwd(pts_local, rotations, plane, grad_out_local)
    else:
        out, g_pts, g_rot, g_plane = fwd_bwd(pts_local, rotations, plane, grad_out_local)
    work = None
    _, world = _rank_world(group)
    if world > 1:
        works = [
            dist.all_reduce(g_plane, group=group, async_op=True),
            dist.all_reduce(g_rot, group=group, async_op=True),
        ]

        class _Pending:
            def wait(self):
                for w_ in works:
                    w_.wait()

        work = _Pending()
        if not async_op:
            work.wait()
            work = None
    return out, g_pts, g_rot, g_plane, work
