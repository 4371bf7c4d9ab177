"""Multi-GPU forms of the hot path: one process per GPU, torch.distributed
(NCCL over NVLink on GPUs; any backend for the host logic).

Neither exists in the reference (quantem-cuda is single-GPU); both follow the
natural sharding of the work:

* TV over D-slabs. Each rank owns a contiguous range of planes of every batch
  slice, stored with one halo plane on each side: ``slab [B, D_local + 2, H, W]``
  (planes 1..D_local owned). The halo planes are filled from the neighbouring
  ranks; the single-sweep kernel then computes the loss terms anchored at
  owned planes and the gradient of owned planes (``tv_loss_3d_slab_cuda``).
  The per-rank sums are added in rank order, so the total is deterministic
  and identical on every rank. Two transports:

  - :class:`PeerSlab` (GPUs of one node): the slab and a small flag block
    live in memory mapped into the neighbours with CUDA IPC. A kernel stores
    the boundary planes straight into the neighbours' halos over NVLink, and
    the loss's finalize kernel stores each rank's fp64 total into every rank
    and adds them in rank order; a step is kernels only, with no library
    collective and no host synchronisation.
  - :func:`exchange_halos` + :func:`tv_loss_slab_fwd_grad`: any
    torch.distributed backend (NCCL send/recv and all_gather, or gloo on CPU).

* K-Planes over points. Each rank evaluates its own points against the
  replicated planes and rotations; point gradients stay local, and the plane
  and rotation gradients are summed over the ranks: by one kernel over peer
  memory (:class:`PeerAllReduce`, deterministic rank-ordered sums) or with a
  torch.distributed all_reduce.

Objects holding peer memory (:class:`PeerSlab`, :class:`PeerAllReduce`) are
collective: every rank creates them together, calls their methods in the
same order on one stream, and calls ``close()`` together before the process
group goes away (a rank must not free memory another rank still maps).

The per-rank compute defaults to the CUDA kernels. ``slab_kernel`` exists so
that the host logic (halo exchange, ownership flags, reductions) can be tested
on CPU ranks with the CPU oracle in place of the device kernel.
"""

from __future__ import annotations

import contextlib
import weakref
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


def _check_neighbour_planes(slab: Tensor, rank: int, world: int, group) -> None:
    """Compares this rank's plane shape (B, H, W) with its neighbours' before
    any plane moves; a mismatch raises ValueError on both sides of it."""
    mine = torch.tensor([slab.shape[0], slab.shape[2], slab.shape[3]], dtype=torch.int64, device=slab.device)
    theirs = {}
    ops = []
    for q in (rank - 1, rank + 1):
        if 0 <= q < world:
            theirs[q] = torch.empty_like(mine)
            ops.append(dist.P2POp(dist.isend, mine, _peer(group, q), group))
            ops.append(dist.P2POp(dist.irecv, theirs[q], _peer(group, q), group))
    for req in dist.batch_isend_irecv(ops):
        req.wait()
    b_h_w = mine.tolist()
    for q, t in theirs.items():
        if t.tolist() != b_h_w:
            raise ValueError(
                f"halo exchange: rank {rank} has planes (B, H, W) = {tuple(b_h_w)} but neighbour "
                f"rank {q} has {tuple(t.tolist())}")


def exchange_halos(slab: Tensor, group=None, check_shapes: bool = True) -> None:
    """Fills the halo planes 0 and -1 of ``slab [B, D_local + 2, H, W]`` with
    the neighbouring ranks' boundary planes (rank r-1's last owned plane and
    rank r+1's first). Ranks at the ends of the global volume leave that halo
    as it is (the kernel is told it is not a neighbour).

    With ``check_shapes`` the neighbours first compare their (B, H, W) and
    raise ValueError on a mismatch (one extra small message each way and a
    host synchronisation); a loop whose shapes are fixed can check once and
    pass False afterwards. A neighbour that never takes part makes the
    exchange fail after the process group's timeout."""
    rank, world = _rank_world(group)
    if world == 1:
        return
    if slab.dim() != 4 or slab.shape[1] < 3:
        raise ValueError(f"slab must be [B, D_local + 2, H, W] with D_local >= 1, got {tuple(slab.shape)}")
    if check_shapes:
        _check_neighbour_planes(slab, rank, world, group)
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
    check_shapes: bool = True,
) -> tuple[Tensor, Tensor]:
    """Loss and gradient of one TV variant over a D-sharded volume.

    Args:
        variant:  SQ, ISO or L1.
        slab:     ``[B, D_local + 2, H, W]`` fp32, owned planes 1..D_local,
                  halos at 0 and D_local + 1 (filled here when ``exchange``).
        grad_out: upstream gradient, shape (1,) (SQ, ISO) or (3,) (L1).
        global_d: D of the whole volume (the isotropic mean divides by the
                  global corner count).
        check_shapes: passed to :func:`exchange_halos`.

    Returns:
        ``(loss, grad)``: the global loss (identical on every rank; the mean
        for ISO, raw sums for SQ and L1) and ``grad [B, D_local + 2, H, W]``
        whose owned planes hold this rank's part of the gradient.
    """
    rank, world = _rank_world(group)
    if exchange:
        exchange_halos(slab, group, check_shapes)
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
    buckets: int | None = None,
    reducer: "PeerAllReduce | None" = None,
    reduce_ctas: int = 32,
):
    """Forward and backward of one K-Planes level over point-sharded ranks.

    Returns ``(out_local, grad_pts_local, grad_rotations, grad_plane, work)``:
    the plane and rotation gradients are summed over ranks with all_reduce
    (``work`` is the pending collective when ``async_op``, so that the next
    level's compute overlaps it; call ``work.wait()`` before reading them).
    ``fwd_bwd(pts, rotations, plane, grad_out) -> (out, g_pts, g_rot, g_plane)``
    replaces the CUDA ops (host-logic tests on CPU ranks).

    On CUDA the planes are converted to channels-last once for both passes.
    ``buckets`` > 1 splits the backward into that many launches over
    consecutive rotations; each bucket's plane gradients are put back in the
    parameter's layout and their all_reduce is enqueued at once, so it runs on
    NCCL's stream while the next bucket's backward computes. Measured on two
    B200s at N = 2^20, T = 4, C = 32, 256^2 the overlap costs more than it
    hides (the collective's SMs and L2 traffic slow the L2-bound backward:
    2.61 ms per step with 4 buckets against 2.16 ms with one), so the default
    there is a single backward launch followed by the all_reduce.

    ``reducer`` (a :func:`kplanes_gradient_reducer` built once per level)
    replaces the NCCL all_reduce: the backward accumulates straight into the
    reducer's peer-memory buffer and one kernel sums it over the ranks in rank
    order (deterministic, identical on every rank); ``work`` is then None.
    With ``buckets`` > 1 the backward runs bucket by bucket over consecutive
    rotations and each bucket's plane gradients are summed on a second stream
    by a kernel of at most ``reduce_ctas`` CTAs while the next bucket's
    backward computes (the rotation gradients go with the last bucket); the
    default there is 4 buckets (at most T), which on eight B200s left 0.21 ms
    of the sum exposed per step against 0.30 ms with one launch.
    """
    _, world = _rank_world(group)
    if buckets is None:
        buckets = 4 if reducer is not None else 1
    if fwd_bwd is None:
        from quantem.cuda.core.ml._ops import _check_kernel_inputs

        _check_kernel_inputs("kplanes_fwd_bwd_sharded", pts_local, rotations, plane, grad_out_local)
    if fwd_bwd is not None:
        out, g_pts, g_rot, g_plane = fwd_bwd(pts_local, rotations, plane, grad_out_local)
        works = []
        if world > 1:
            works = [
                dist.all_reduce(g_plane, group=group, async_op=True),
                dist.all_reduce(g_rot, group=group, async_op=True),
            ]
    elif reducer is not None:
        out, g_pts, g_rot, g_plane = _kplanes_fwd_bwd_peer(pts_local, rotations, plane, grad_out_local, reducer,
                                                           buckets, reduce_ctas)
        works = []
    else:
        out, g_pts, g_rot, g_plane, works = _kplanes_fwd_bwd_bucketed(
            pts_local, rotations, plane, grad_out_local, group, world, buckets)
    work = None
    if works:

        class _Pending:
            def wait(self):
                for w_ in works:
                    w_.wait()

        work = _Pending()
        if not async_op:
            work.wait()
            work = None
    return out, g_pts, g_rot, g_plane, work


def _rotation_buckets(t_count: int, buckets: int) -> list[tuple[int, int]]:
    """Consecutive rotation ranges, as equal as possible, at most ``buckets``."""
    k = max(1, min(int(buckets), t_count))
    edges = [t_count * i // k for i in range(k + 1)]
    return [(a, b) for a, b in zip(edges[:-1], edges[1:]) if b > a]


def _kplanes_fwd_bwd_peer(pts, rotations, plane, grad_out, reducer, buckets=1, reduce_ctas=32):
    from quantem.cuda import _core
    from quantem.cuda.core.ml._ops import _channels_last, _from_channels_last

    dev = pts.device
    p = pts.contiguous()
    r = rotations.contiguous()
    t_count = r.shape[0]
    c, h, w = plane.shape[1:]
    n = p.shape[0]
    P = plane.numel()
    if reducer.numel < P + r.numel():
        raise ValueError(f"reducer holds {reducer.numel} floats; the gradients need {P + r.numel()}")
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        g = _channels_last(plane, stream)
        out = torch.empty((n, t_count * c), dtype=torch.float32, device=dev)
        _core.kplanes_tilted_fuse_cuda(p.data_ptr(), r.data_ptr(), g.data_ptr(), out.data_ptr(),
                                       n, t_count, c, h, w, stream)
        gout = grad_out.detach().to(dtype=torch.float32, device=dev).contiguous()
        g_pts = torch.zeros_like(p)
        buf = reducer.buffer
        buf[: P + r.numel()].zero_()
        g_cl = buf[:P].view(3 * t_count, h, w, c)
        g_rot = buf[P : P + r.numel()].view(t_count, 3, 3)
        ranges = _rotation_buckets(t_count, buckets)
        if len(ranges) == 1:
            _core.kplanes_tilted_fuse_grad_cuda(p.data_ptr(), r.data_ptr(), g.data_ptr(), gout.data_ptr(),
                                                g_cl.data_ptr(), g_rot.data_ptr(), g_pts.data_ptr(),
                                                n, t_count, c, h, w, stream)
            reducer.all_reduce(0, P + r.numel())
        else:
            # bucket k's planes 3*t0 .. 3*t1-1 are floats [3*t0*hwc, 3*t1*hwc)
            # of the channels-last gradient; the last bucket's range runs on
            # through the rotation gradient, complete only after every bucket
            main = torch.cuda.current_stream(dev)
            side = reducer.side_stream()
            per_rot = 3 * h * w * c
            for k, (t0, t1) in enumerate(ranges):
                _core.kplanes_tilted_fuse_grad_rotations_cuda(
                    p.data_ptr(), r.data_ptr(), g.data_ptr(), gout.data_ptr(), g_cl.data_ptr(),
                    g_rot.data_ptr(), g_pts.data_ptr(), n, t_count, c, h, w, t0, t1, stream)
                done = torch.cuda.Event()
                done.record(main)
                side.wait_event(done)
                last = k == len(ranges) - 1
                end = P + r.numel() if last else t1 * per_rot
                reducer.all_reduce(t0 * per_rot, end - t0 * per_rot, 0 if last else reduce_ctas, stream=side)
            main.wait_stream(side)
        # the reducer's buffer is reused by the next call: hand out copies
        g_plane = _from_channels_last(g_cl, plane, stream)
        if g_plane.data_ptr() == g_cl.data_ptr():
            g_plane = g_plane.clone(memory_format=torch.channels_last)
        g_rot = g_rot.clone()
    return out, g_pts, g_rot, g_plane


def _kplanes_fwd_bwd_bucketed(pts, rotations, plane, grad_out, group, world, buckets=1):
    from quantem.cuda import _core
    from quantem.cuda.core.ml._ops import _channels_last

    dev = pts.device
    p = pts.contiguous()
    r = rotations.contiguous()
    t_count = r.shape[0]
    c, h, w = plane.shape[1:]
    n = p.shape[0]
    stream = torch.cuda.current_stream(dev).cuda_stream
    works = []
    with torch.cuda.device(dev):
        g = _channels_last(plane, stream)
        out = torch.empty((n, t_count * c), dtype=torch.float32, device=dev)
        _core.kplanes_tilted_fuse_cuda(p.data_ptr(), r.data_ptr(), g.data_ptr(), out.data_ptr(),
                                       n, t_count, c, h, w, stream)
        gout = grad_out.detach().to(dtype=torch.float32, device=dev).contiguous()
        g_pts = torch.zeros_like(p)
        g_rot = torch.zeros_like(r)
        g_cl = torch.zeros(g.shape, dtype=torch.float32, device=dev)
        keep_cl = plane.permute(0, 2, 3, 1).is_contiguous()
        g_plane = g_cl.permute(0, 3, 1, 2) if keep_cl else torch.empty(
            (3 * t_count, c, h, w), dtype=torch.float32, device=dev)
        nb = max(1, min(int(buckets), t_count))
        bounds = [t_count * k // nb for k in range(nb + 1)]
        for t0, t1 in zip(bounds[:-1], bounds[1:]):
            if t0 == t1:
                continue
            _core.kplanes_tilted_fuse_grad_rotations_cuda(
                p.data_ptr(), r.data_ptr(), g.data_ptr(), gout.data_ptr(), g_cl.data_ptr(),
                g_rot.data_ptr(), g_pts.data_ptr(), n, t_count, c, h, w, t0, t1, stream)
            if keep_cl:
                bucket = g_cl[3 * t0 : 3 * t1]
            else:
                bucket = g_plane[3 * t0 : 3 * t1]
                _core.kplanes_planes_from_channels_last_cuda(g_cl[3 * t0].data_ptr(), bucket.data_ptr(),
                                                             3 * (t1 - t0), c, h, w, stream)
            if world > 1:
                works.append(dist.all_reduce(bucket, group=group, async_op=True))
        if world > 1:
            works.append(dist.all_reduce(g_rot, group=group, async_op=True))
    return out, g_pts, g_rot, g_plane, works


# ── D-slabs over peer memory ────────────────────────────────────────────────


@contextlib.contextmanager
def _unmap_on_error(mapped: list[int]):
    """Closes the peer mappings opened so far if opening the rest fails (the
    other ranks then fail at the constructor's barrier, after the process
    group's timeout)."""
    from quantem.cuda import _core

    try:
        yield
    except BaseException:
        for ptr in mapped:
            try:
                _core.ipc_close(ptr)
            except RuntimeError:
                pass
        mapped.clear()
        raise


def _same_on_every_rank(values: list, what: str) -> None:
    """Raises ValueError (on every rank, which all hold the same gathered
    list) unless every rank passed the same value."""
    if any(v != values[0] for v in values):
        raise ValueError(f"{what} differs between ranks: " + ", ".join(f"rank {q}: {v}" for q, v in enumerate(values)))


class _PeerAllocation:
    """One ``quantem_cuda_peer_alloc`` allocation (zero-filled, IPC-exportable),
    viewable as a torch tensor through ``__cuda_array_interface__``; freed when
    the last tensor viewing it is gone."""

    def __init__(self, shape: tuple[int, ...], typestr: str, itemsize: int, device: torch.device):
        from quantem.cuda import _core

        n = 1
        for d in shape:
            n *= int(d)
        self.device = device
        with torch.cuda.device(device):
            self.ptr = int(_core.peer_alloc(max(1, n * itemsize)))
        self.__cuda_array_interface__ = {
            "shape": tuple(int(d) for d in shape),
            "typestr": typestr,
            "data": (self.ptr, False),
            "version": 3,
            "strides": None,
            "stream": None,
        }
        self._finalizer = weakref.finalize(self, _free_peer, self.ptr, device)


def _free_peer(ptr: int, device: torch.device) -> None:
    from quantem.cuda import _core

    with torch.cuda.device(device):
        _core.peer_free(ptr)


class PeerSlab:
    """This rank's D-slab of a ``[B, global_d, H, W]`` volume, with its halo
    planes and loss sums exchanged over peer memory (CUDA IPC on the GPUs of
    one node, stores over NVLink).

    ``slab`` is ``[B, D_local + 2, H, W]``; write the owned planes
    (``owned``, global planes ``d_lo..d_hi-1``) and call :meth:`fwd_grad`.
    Every rank of ``group`` must construct it together and make the same calls
    in the same order, on one stream per rank. A wait for another rank gives
    up after ``timeout_s`` (the loss becomes NaN and the device fault word
    gets ``FAULT_PEER_WAIT``) instead of hanging.
    """

    def __init__(self, batch: int, global_d: int, height: int, width: int, group=None,
                 device: torch.device | None = None, timeout_s: float = 10.0):
        from quantem.cuda import _core

        rank, world = _rank_world(group)
        if world > _core.MAX_PEER_RANKS:
            raise ValueError(f"PeerSlab supports at most {_core.MAX_PEER_RANKS} ranks, got {world}")
        lo, hi = slab_bounds(global_d, rank, world)
        if hi - lo < 1:
            raise ValueError(f"global_d={global_d} leaves rank {rank} of {world} without planes")
        self.group, self.rank, self.world = group, rank, world
        self.global_d, self.d_lo, self.d_hi = global_d, lo, hi
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        dp = hi - lo + 2
        self.shape = (batch, dp, height, width)
        self._slab_mem = _PeerAllocation(self.shape, "<f4", 4, self.device)
        self._comm_mem = _PeerAllocation((int(_core.tv_peer_comm_bytes()),), "|u1", 1, self.device)
        self.slab = torch.as_tensor(self._slab_mem, device=self.device)
        with torch.cuda.device(self.device):
            mine = ((batch, global_d, height, width), dp, _core.ipc_handle(self._slab_mem.ptr),
                    _core.ipc_handle(self._comm_mem.ptr))
        infos = [None] * world
        dist.all_gather_object(infos, mine, group=group)
        # the neighbours' halo stores are sized by this rank's (B, H, W): every
        # rank must describe the same volume before any memory is mapped
        _same_on_every_rank([i[0] for i in infos], "PeerSlab (batch, global_d, height, width)")
        self._mapped: list[int] = []
        comm, prev_ptr, prev_dp, next_ptr, next_dp = [], 0, 0, 0, 0
        with torch.cuda.device(self.device), _unmap_on_error(self._mapped):
            for q, (_, dq, slab_h, comm_h) in enumerate(infos):
                if q == rank:
                    comm.append(self._comm_mem.ptr)
                    continue
                c = int(_core.ipc_open(comm_h))
                self._mapped.append(c)
                comm.append(c)
                if q == rank - 1 or q == rank + 1:
                    sp = int(_core.ipc_open(slab_h))
                    self._mapped.append(sp)
                    if q == rank - 1:
                        prev_ptr, prev_dp = sp, dq
                    else:
                        next_ptr, next_dp = sp, dq
        self._peers = _core.TvPeers(rank, world, int(timeout_s * 1e9), comm, prev_ptr, prev_dp,
                                    next_ptr, next_dp)
        from quantem.cuda._common import _workspace

        self._ws = _workspace(self.device)
        self._ws_many = []
        self._halo_seq = 0
        self._red_seq = 0
        dist.barrier(group=group)

    @property
    def owned(self) -> Tensor:
        """The owned planes, ``slab[:, 1:-1]`` (a view)."""
        return self.slab[:, 1:-1]

    def exchange_halos(self) -> None:
        """Fills the halo planes from the neighbours (kernel on the current
        stream; returns at once)."""
        from quantem.cuda import _core

        self._halo_seq += 1
        b, dp, h, w = self.shape
        with torch.cuda.device(self.device):
            _core.tv_slab_halo_exchange_cuda(self._peers, self._halo_seq, self._slab_mem.ptr, b, dp, h, w,
                                             torch.cuda.current_stream(self.device).cuda_stream)

    def fwd_grad(self, variant: int, grad_out: Tensor, eps: float = 1e-8, grad: Tensor | None = None,
                 exchange: bool = True) -> tuple[Tensor, Tensor]:
        """Global loss and this rank's gradient for one TV variant (the same
        contract as :func:`tv_loss_slab_fwd_grad`). ``grad`` (``slab``'s shape)
        is written if given; its owned planes receive the gradient."""
        from quantem.cuda import _core

        halo_seq = 0
        if exchange:
            # done inside the sweep kernel (no separate launch)
            self._halo_seq += 1
            halo_seq = self._halo_seq
        b, dp, h, w = self.shape
        scale = 1.0
        if variant == ISO:
            scale = 1.0 / max(1, b * (self.global_d - 1) * (h - 1) * (w - 1))
        if grad is None:
            grad = torch.empty(self.shape, dtype=torch.float32, device=self.device)
        elif tuple(grad.shape) != self.shape or not grad.is_contiguous() or grad.dtype != torch.float32:
            raise ValueError(f"grad must be a contiguous fp32 tensor of shape {self.shape}")
        g = grad_out.to(device=self.device, dtype=torch.float32).contiguous()
        if g.numel() != _N_ACC[variant]:
            raise ValueError(f"grad_out needs {_N_ACC[variant]} element(s), got {g.numel()}")
        acc = torch.empty(_N_ACC[variant], dtype=torch.float32, device=self.device)
        self._red_seq += 1
        with torch.cuda.device(self.device):
            _core.tv_loss_3d_slab_peer_cuda(
                self._peers, halo_seq, self._red_seq, variant, _LOSS | _GRAD | _OVERWRITE, self._slab_mem.ptr,
                g.data_ptr(), acc.data_ptr(), grad.data_ptr(), b, dp, h, w, 1, dp - 1,
                int(self.rank > 0), int(self.rank < self.world - 1), float(eps), float(scale),
                self._ws.data_ptr(), self._ws.numel(), torch.cuda.current_stream(self.device).cuda_stream)
        return (acc.squeeze(0) if variant != L1 else acc), grad

    def fwd_grad_many(self, terms, exchange: bool = True, grads=None):
        """Several losses of one step over the same slab with a single
        cross-rank wait: ``terms`` is a list of ``(variant, grad_out, eps)``;
        each sweep writes its own gradient (``grads[k]`` if given), and one
        finalize kernel adds every loss over the ranks in rank order. Returns
        ``[(loss, grad), ...]`` in the order of ``terms``. The halos are
        exchanged by the first sweep when ``exchange``."""
        from quantem.cuda import _core
        from quantem.cuda._common import _workspace

        b, dp, h, w = self.shape
        if not 1 <= len(terms) <= 8 or sum(_N_ACC[t[0]] for t in terms) > 8:
            raise ValueError("fwd_grad_many takes 1..8 terms with at most 8 loss sums in total")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if len(self._ws_many) < len(terms):
            self._ws_many += [_workspace(self.device) for _ in range(len(terms) - len(self._ws_many))]
        fin, out = [], []
        with torch.cuda.device(self.device):
            for k, (variant, grad_out, eps) in enumerate(terms):
                halo_seq = 0
                if exchange and k == 0:
                    self._halo_seq += 1
                    halo_seq = self._halo_seq
                scale = 1.0
                if variant == ISO:
                    scale = 1.0 / max(1, b * (self.global_d - 1) * (h - 1) * (w - 1))
                grad = None if grads is None else grads[k]
                if grad is None:
                    grad = torch.empty(self.shape, dtype=torch.float32, device=self.device)
                elif tuple(grad.shape) != self.shape or not grad.is_contiguous() or grad.dtype != torch.float32:
                    raise ValueError(f"grads[{k}] must be a contiguous fp32 tensor of shape {self.shape}")
                g = grad_out.to(device=self.device, dtype=torch.float32).contiguous()
                if g.numel() != _N_ACC[variant]:
                    raise ValueError(f"grad_out needs {_N_ACC[variant]} element(s), got {g.numel()}")
                acc = torch.empty(_N_ACC[variant], dtype=torch.float32, device=self.device)
                ws = self._ws_many[k]
                n = _core.tv_loss_3d_slab_sweep_cuda(
                    self._peers, halo_seq, variant, _LOSS | _GRAD, self._slab_mem.ptr, g.data_ptr(),
                    grad.data_ptr(), b, dp, h, w, 1, dp - 1, int(self.rank > 0),
                    int(self.rank < self.world - 1), float(eps), float(scale), ws.data_ptr(), ws.numel(),
                    stream)
                fin.append((ws.data_ptr(), n, _N_ACC[variant], acc.data_ptr(), float(scale), True))
                out.append(((acc.squeeze(0) if variant != L1 else acc), grad))
            self._red_seq += 1
            _core.tv_loss_3d_peer_finalize_cuda(self._peers, self._red_seq, fin, stream)
        return out

    def close(self) -> None:
        """Unmaps the peers' memory after every rank has finished with it.
        Collective: every rank calls it."""
        from quantem.cuda import _core

        if self._mapped is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._mapped:
                _core.ipc_close(p)
        self._mapped = None
        dist.barrier(group=self.group)


class PeerAllReduce:
    """A float32 buffer of ``numel`` elements on every rank, summed over the
    ranks in place by one kernel over peer memory (CUDA IPC on the GPUs of one
    node): rank r adds chunk r of all buffers in rank order and stores it into
    every buffer, so the result is bitwise identical on every rank and from
    run to run. Every rank constructs it together and calls :meth:`all_reduce`
    in the same order (one stream per rank)."""

    def __init__(self, numel: int, group=None, device: torch.device | None = None, timeout_s: float = 10.0):
        from quantem.cuda import _core

        rank, world = _rank_world(group)
        if world > _core.MAX_PEER_RANKS:
            raise ValueError(f"PeerAllReduce supports at most {_core.MAX_PEER_RANKS} ranks, got {world}")
        self.group, self.rank, self.world, self.numel = group, rank, world, int(numel)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._buf_mem = _PeerAllocation((self.numel,), "<f4", 4, self.device)
        self._comm_mem = _PeerAllocation((int(_core.peer_allreduce_comm_bytes()),), "|u1", 1, self.device)
        self.buffer = torch.as_tensor(self._buf_mem, device=self.device)
        with torch.cuda.device(self.device):
            mine = (self.numel, _core.ipc_handle(self._buf_mem.ptr), _core.ipc_handle(self._comm_mem.ptr))
        infos = [None] * world
        dist.all_gather_object(infos, mine, group=group)
        # each rank reads and writes every buffer over its whole length
        _same_on_every_rank([i[0] for i in infos], "PeerAllReduce numel")
        self._mapped: list[int] = []
        bufs, comms = [], []
        with torch.cuda.device(self.device), _unmap_on_error(self._mapped):
            for q, (_, buf_h, comm_h) in enumerate(infos):
                if q == rank:
                    bufs.append(self._buf_mem.ptr)
                    comms.append(self._comm_mem.ptr)
                    continue
                b = int(_core.ipc_open(buf_h))
                c = int(_core.ipc_open(comm_h))
                self._mapped += [b, c]
                bufs.append(b)
                comms.append(c)
        self._group = _core.PeerGroup(rank, world, int(timeout_s * 1e9), comms, bufs)
        self._seq = 0
        self._side: torch.cuda.Stream | None = None
        dist.barrier(group=group)

    def side_stream(self) -> torch.cuda.Stream:
        """A stream of this reducer's own, for sums that overlap other work."""
        if self._side is None:
            self._side = torch.cuda.Stream(device=self.device)
        return self._side

    def all_reduce(self, offset: int = 0, count: int | None = None, max_ctas: int = 0,
                   stream: torch.cuda.Stream | None = None) -> Tensor:
        """Sums ``buffer[offset : offset + count]`` (all of it by default) over
        the ranks in place, by one kernel of at most ``max_ctas`` CTAs (0: two
        per SM) on ``stream`` (default: the current stream), and returns that
        range. Every rank makes the same calls in the same order."""
        from quantem.cuda import _core

        count = self.numel - offset if count is None else int(count)
        if offset < 0 or count < 0 or offset + count > self.numel:
            raise ValueError(f"PeerAllReduce.all_reduce: range [{offset}, {offset + count}) outside the "
                             f"buffer of {self.numel} floats")
        if max_ctas < 0:
            raise ValueError(f"PeerAllReduce.all_reduce: max_ctas must be >= 0, got {max_ctas}")
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        self._seq += 1
        with torch.cuda.device(self.device):
            _core.peer_allreduce_sum_f32_range_cuda(self._group, self._seq, int(offset), count, int(max_ctas),
                                                    st.cuda_stream)
        return self.buffer[offset : offset + count]

    def close(self) -> None:
        """Unmaps the peers' buffers (collective)."""
        from quantem.cuda import _core

        if self._mapped is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._mapped:
                _core.ipc_close(p)
        self._mapped = None
        dist.barrier(group=self.group)


def kplanes_gradient_reducer(plane: Tensor, rotations: Tensor, group=None) -> PeerAllReduce:
    """A :class:`PeerAllReduce` sized for one K-Planes level's plane and
    rotation gradients (``3T·H·W·C + 9T`` floats), for
    :func:`kplanes_fwd_bwd_sharded`'s ``reducer``."""
    n = plane.numel() + rotations.numel()
    return PeerAllReduce(n, group=group, device=plane.device)
