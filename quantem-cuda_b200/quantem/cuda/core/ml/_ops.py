"""torch registration of the fused tilted K-Planes kernels.

Mirrors the reference's src/quantem/cuda/core/ml/_ops.py for the hot path
(same op names, schemas, fake implementations, autograd wiring, public wrapper
and validation messages):

    quantem_cuda::kplanes_tilted_fuse(Tensor pts, Tensor rotations, Tensor plane) -> Tensor
                                                                          (:28-47)
    quantem_cuda::kplanes_tilted_fuse_bwd(pts, rotations, plane, grad_out) -> Tensor[]
                                                                          (:50-101)

The kernels read the planes channels-last ``[3T, H, W, C]``. Where the
reference permutes with torch on every call (:21-25, :82), this layer uses the
library's own transpose kernels, and skips the copy entirely when ``plane`` is
already stored channels-last (``plane.permute(0, 2, 3, 1).is_contiguous()``,
e.g. a parameter created with ``memory_format=torch.channels_last``); the
plane gradient is then returned with the parameter's own strides.

The public wrappers call the ops' implementations through
``torch.autograd.Function`` classes when they run eagerly on plain tensors
(``_eager``): the torch.library dispatcher costs tens of microseconds of host
time per call, as much as a small point set's kernels. Under
``torch.compile`` and for tensor subclasses the registered ops run unchanged.
"""

from __future__ import annotations

import torch
from torch import Tensor

from quantem.cuda import _core
from quantem.cuda.core._ops import _eager, _on_device


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _channels_last(plane: Tensor, stream: int) -> Tensor:
    """(3T, C, H, W) → contiguous (3T, H, W, C); free when already stored so."""
    cl = plane.permute(0, 2, 3, 1)
    if cl.is_contiguous():
        return cl
    src = plane.contiguous()
    n, c, h, w = src.shape
    dst = torch.empty((n, h, w, c), dtype=src.dtype, device=src.device)
    _core.kplanes_planes_to_channels_last_cuda(src.data_ptr(), dst.data_ptr(), n, c, h, w, stream)
    return dst


def _check_kernel_inputs(fn: str, pts: Tensor, rotations: Tensor, plane: Tensor,
                         grad_out: Tensor | None = None, taps: int = 1) -> None:
    """Checks what the kernels index by: the op layer passes raw device
    pointers, so a plane count, an upstream-gradient size or a device that
    does not match would make a kernel read outside its buffers. Raises
    ValueError / TypeError (the public wrappers check more, with the
    reference's messages, before reaching here)."""
    if pts.ndim != 2 or pts.shape[-1] != 3:
        raise ValueError(f"{fn}: pts must be [B, 3], got {tuple(pts.shape)}")
    if rotations.ndim != 3 or tuple(rotations.shape[-2:]) != (3, 3):
        raise ValueError(f"{fn}: rotations must be [T, 3, 3], got {tuple(rotations.shape)}")
    t = rotations.shape[0]
    if plane.ndim != 4 or plane.shape[0] != 3 * t:
        raise ValueError(f"{fn}: plane must be [3*T, C, H, W] with T={t}, got {tuple(plane.shape)}")
    for name, x in (("pts", pts), ("rotations", rotations), ("plane", plane)):
        if x.dtype != torch.float32:
            raise TypeError(f"{fn}: {name} must be fp32, got {x.dtype}")
        if not x.is_cuda or x.device != pts.device:
            raise ValueError(f"{fn}: {name} is on {x.device}; all inputs must be on {pts.device} (CUDA)")
    if grad_out is not None:
        want = taps * pts.shape[0] * t * plane.shape[1]
        if grad_out.numel() != want:
            shape = (pts.shape[0], t * plane.shape[1]) if taps == 1 else (taps, pts.shape[0], t * plane.shape[1])
            raise ValueError(f"{fn}: grad_out must have shape {shape}, got {tuple(grad_out.shape)}")


def _from_channels_last(grad_cl: Tensor, like: Tensor, stream: int) -> Tensor:
    """(3T, H, W, C) → a (3T, C, H, W) tensor with ``like``'s memory layout."""
    if like.permute(0, 2, 3, 1).is_contiguous():
        return grad_cl.permute(0, 3, 1, 2)
    n, h, w, c = grad_cl.shape
    dst = torch.empty((n, c, h, w), dtype=grad_cl.dtype, device=grad_cl.device)
    _core.kplanes_planes_from_channels_last_cuda(grad_cl.data_ptr(), dst.data_ptr(), n, c, h, w, stream)
    return dst


# ── fused TILTED K-Planes interpolation ───────────────────────────────────


def _kpt_fwd_impl(pts: Tensor, rotations: Tensor, plane: Tensor) -> Tensor:
    _check_kernel_inputs("kplanes_tilted_fuse", pts, rotations, plane)
    p = pts.contiguous()
    r = rotations.contiguous()
    c, h, w = plane.shape[1:]
    b = p.shape[0]
    t = r.shape[0]
    stream = _stream(p.device)
    with _on_device(p.device):
        g = _channels_last(plane, stream)
        out = torch.empty((b, t * c), dtype=torch.float32, device=p.device)
        _core.kplanes_tilted_fuse_cuda(
            p.data_ptr(), r.data_ptr(), g.data_ptr(), out.data_ptr(), b, t, c, h, w, stream
        )
    return out


@torch.library.custom_op("quantem_cuda::kplanes_tilted_fuse", mutates_args=())
def _kplanes_tilted_fuse(pts: Tensor, rotations: Tensor, plane: Tensor) -> Tensor:
    return _kpt_fwd_impl(pts, rotations, plane)


@_kplanes_tilted_fuse.register_fake
def _(pts: Tensor, rotations: Tensor, plane: Tensor) -> Tensor:
    return pts.new_empty((pts.shape[0], rotations.shape[0] * plane.shape[1]))


def _kpt_bwd_impl(pts: Tensor, rotations: Tensor, plane: Tensor, grad_out: Tensor) -> list[Tensor]:
    _check_kernel_inputs("kplanes_tilted_fuse_bwd", pts, rotations, plane, grad_out)
    p = pts.contiguous()
    r = rotations.contiguous()
    c, h, w = plane.shape[1:]
    b = p.shape[0]
    t = r.shape[0]
    stream = _stream(p.device)
    with _on_device(p.device):
        g = _channels_last(plane, stream)
        gout = grad_out.detach().to(dtype=torch.float32, device=p.device).contiguous()
        grad_pts = torch.zeros_like(p)
        grad_r = torch.zeros_like(r)
        grad_plane_cl = torch.zeros(g.shape, dtype=torch.float32, device=p.device)
        _core.kplanes_tilted_fuse_grad_cuda(
            p.data_ptr(),
            r.data_ptr(),
            g.data_ptr(),
            gout.data_ptr(),
            grad_plane_cl.data_ptr(),
            grad_r.data_ptr(),
            grad_pts.data_ptr(),
            b,
            t,
            c,
            h,
            w,
            stream,
        )
        grad_plane = _from_channels_last(grad_plane_cl, plane, stream)
    return [grad_pts, grad_r, grad_plane]


@torch.library.custom_op("quantem_cuda::kplanes_tilted_fuse_bwd", mutates_args=())
def _kplanes_tilted_fuse_bwd(
    pts: Tensor, rotations: Tensor, plane: Tensor, grad_out: Tensor
) -> list[Tensor]:
    return _kpt_bwd_impl(pts, rotations, plane, grad_out)


@_kplanes_tilted_fuse_bwd.register_fake
def _(pts: Tensor, rotations: Tensor, plane: Tensor, grad_out: Tensor) -> list[Tensor]:
    return [torch.empty_like(pts), torch.empty_like(rotations), torch.empty_like(plane)]


def _kpt_setup_context(ctx, inputs, output) -> None:
    pts, rotations, plane = inputs
    ctx.save_for_backward(pts, rotations, plane)


def _kpt_backward(ctx, grad_out):
    pts, rotations, plane = ctx.saved_tensors
    grad_pts, grad_r, grad_plane = _kplanes_tilted_fuse_bwd(pts, rotations, plane, grad_out)
    return grad_pts, grad_r, grad_plane


_kplanes_tilted_fuse.register_autograd(_kpt_backward, setup_context=_kpt_setup_context)


class _KPlanesTilted(torch.autograd.Function):
    """The same forward and backward as the registered op, for eager calls on
    plain tensors: no torch.library dispatch on the way (see ``_eager``)."""

    @staticmethod
    def forward(ctx, pts: Tensor, rotations: Tensor, plane: Tensor) -> Tensor:
        ctx.save_for_backward(pts, rotations, plane)
        return _kpt_fwd_impl(pts, rotations, plane)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad_out):
        pts, rotations, plane = ctx.saved_tensors
        grad_pts, grad_r, grad_plane = _kpt_bwd_impl(pts, rotations, plane, grad_out)
        return grad_pts, grad_r, grad_plane


# ── several levels in one launch ──────────────────────────────────────────
#
# A multiscale encoder samples the same points under the same rotations at
# every level (each level's planes at their own resolution). One launch per
# pass covers all levels: level l's output is kplanes_tilted_fuse(pts,
# rotations, planes[l]) bit for bit, and the backward adds every level's
# point and rotation gradients into one sum.


def _check_levels(fn: str, pts: Tensor, rotations: Tensor, planes: list[Tensor],
                  grad_outs: list[Tensor] | None = None) -> None:
    if not 1 <= len(planes) <= _core.KP_MAX_LEVELS:
        raise ValueError(f"{fn}: 1 to {_core.KP_MAX_LEVELS} levels, got {len(planes)}")
    c = planes[0].shape[1] if planes[0].ndim == 4 else -1
    for lv, plane in enumerate(planes):
        _check_kernel_inputs(fn, pts, rotations, plane,
                             None if grad_outs is None else grad_outs[lv])
        if plane.shape[1] != c:
            raise ValueError(f"{fn}: every level needs the same channel count C, got {c} and "
                             f"{plane.shape[1]} (level {lv})")
    if grad_outs is not None and len(grad_outs) != len(planes):
        raise ValueError(f"{fn}: one grad_out per level, got {len(grad_outs)} for {len(planes)} levels")


def _kpl_fwd_impl(pts: Tensor, rotations: Tensor, planes: list[Tensor]) -> list[Tensor]:
    _check_levels("kplanes_tilted_fuse_levels", pts, rotations, planes)
    p = pts.contiguous()
    r = rotations.contiguous()
    b, t = p.shape[0], r.shape[0]
    c = planes[0].shape[1]
    stream = _stream(p.device)
    with _on_device(p.device):
        grids = [_channels_last(plane, stream) for plane in planes]
        outs = [torch.empty((b, t * c), dtype=torch.float32, device=p.device) for _ in planes]
        _core.kplanes_tilted_fuse_levels_cuda(
            p.data_ptr(), r.data_ptr(), [g.data_ptr() for g in grids], [o.data_ptr() for o in outs],
            [pl.shape[2] for pl in planes], [pl.shape[3] for pl in planes], b, t, c, stream,
        )
    return outs


@torch.library.custom_op("quantem_cuda::kplanes_tilted_fuse_levels", mutates_args=())
def _kplanes_tilted_fuse_levels(pts: Tensor, rotations: Tensor, planes: list[Tensor]) -> list[Tensor]:
    return _kpl_fwd_impl(pts, rotations, planes)


@_kplanes_tilted_fuse_levels.register_fake
def _(pts: Tensor, rotations: Tensor, planes: list[Tensor]) -> list[Tensor]:
    return [pts.new_empty((pts.shape[0], rotations.shape[0] * pl.shape[1])) for pl in planes]


def _kpl_bwd_impl(pts: Tensor, rotations: Tensor, planes: list[Tensor], grad_outs: list[Tensor]) -> list[Tensor]:
    """[grad_pts, grad_rotations, grad_plane_0, ..., grad_plane_{L-1}]"""
    _check_levels("kplanes_tilted_fuse_levels_bwd", pts, rotations, planes, grad_outs)
    p = pts.contiguous()
    r = rotations.contiguous()
    b, t = p.shape[0], r.shape[0]
    c = planes[0].shape[1]
    stream = _stream(p.device)
    with _on_device(p.device):
        grids = [_channels_last(plane, stream) for plane in planes]
        gouts = [go.detach().to(dtype=torch.float32, device=p.device).contiguous() for go in grad_outs]
        grad_pts = torch.zeros_like(p)
        grad_r = torch.zeros_like(r)
        grads_cl = [torch.zeros(g.shape, dtype=torch.float32, device=p.device) for g in grids]
        _core.kplanes_tilted_fuse_levels_grad_cuda(
            p.data_ptr(), r.data_ptr(), [g.data_ptr() for g in grids], [go.data_ptr() for go in gouts],
            [gc.data_ptr() for gc in grads_cl], [pl.shape[2] for pl in planes], [pl.shape[3] for pl in planes],
            grad_r.data_ptr(), grad_pts.data_ptr(), b, t, c, stream,
        )
        grad_planes = [_from_channels_last(gc, pl, stream) for gc, pl in zip(grads_cl, planes)]
    return [grad_pts, grad_r, *grad_planes]


@torch.library.custom_op("quantem_cuda::kplanes_tilted_fuse_levels_bwd", mutates_args=())
def _kplanes_tilted_fuse_levels_bwd(
    pts: Tensor, rotations: Tensor, planes: list[Tensor], grad_outs: list[Tensor]
) -> list[Tensor]:
    """[grad_pts, grad_rotations, grad_plane_0, ..., grad_plane_{L-1}]"""
    return _kpl_bwd_impl(pts, rotations, planes, grad_outs)


@_kplanes_tilted_fuse_levels_bwd.register_fake
def _(pts: Tensor, rotations: Tensor, planes: list[Tensor], grad_outs: list[Tensor]) -> list[Tensor]:
    return [torch.empty_like(pts), torch.empty_like(rotations), *[torch.empty_like(pl) for pl in planes]]


def _kpl_setup_context(ctx, inputs, output) -> None:
    pts, rotations, planes = inputs
    ctx.n_levels = len(planes)
    ctx.save_for_backward(pts, rotations, *planes)


def _kpl_backward(ctx, grad_outs):
    pts, rotations, *planes = ctx.saved_tensors
    gouts = [go if go is not None else torch.zeros((pts.shape[0], rotations.shape[0] * pl.shape[1]),
                                                   dtype=torch.float32, device=pts.device)
             for go, pl in zip(grad_outs, planes)]
    grad_pts, grad_r, *grad_planes = _kplanes_tilted_fuse_levels_bwd(pts, rotations, planes, gouts)
    return grad_pts, grad_r, grad_planes


_kplanes_tilted_fuse_levels.register_autograd(_kpl_backward, setup_context=_kpl_setup_context)


class _KPlanesTiltedLevels(torch.autograd.Function):
    """Eager counterpart of the registered multi-level op (see
    ``_KPlanesTilted``); the planes come as separate arguments. A level whose
    output takes no part in the loss gets a zero upstream gradient."""

    @staticmethod
    def forward(ctx, pts: Tensor, rotations: Tensor, *planes: Tensor):
        ctx.save_for_backward(pts, rotations, *planes)
        return tuple(_kpl_fwd_impl(pts, rotations, list(planes)))

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, *grad_outs):
        pts, rotations, *planes = ctx.saved_tensors
        grad_pts, grad_r, *grad_planes = _kpl_bwd_impl(pts, rotations, planes, list(grad_outs))
        return (grad_pts, grad_r, *grad_planes)


# ── four-tap variant for finite-difference TV regularisation ──────────────
#
# The reference's kplanes_tilted_tv_fuse (core/ml/_ops.py:103-204): tap 0 at
# R·x (the base op's values, bit for bit), taps 1..3 at R·x + h·R[:, k-1];
# output [4, B, T*C] with the tap outermost; h carries no gradient.


def _kpt_tv_fwd_impl(pts: Tensor, rotations: Tensor, plane: Tensor, h: float) -> Tensor:
    _check_kernel_inputs("kplanes_tilted_tv_fuse", pts, rotations, plane)
    p = pts.contiguous()
    r = rotations.contiguous()
    c, hh, w = plane.shape[1:]
    b = p.shape[0]
    t = r.shape[0]
    stream = _stream(p.device)
    with _on_device(p.device):
        g = _channels_last(plane, stream)
        out = torch.empty((4, b, t * c), dtype=torch.float32, device=p.device)
        _core.kplanes_tilted_tv_fuse_cuda(
            p.data_ptr(), r.data_ptr(), g.data_ptr(), out.data_ptr(), b, t, c, hh, w, float(h), stream
        )
    return out


@torch.library.custom_op("quantem_cuda::kplanes_tilted_tv_fuse", mutates_args=())
def _kplanes_tilted_tv_fuse(pts: Tensor, rotations: Tensor, plane: Tensor, h: float) -> Tensor:
    return _kpt_tv_fwd_impl(pts, rotations, plane, h)


@_kplanes_tilted_tv_fuse.register_fake
def _(pts: Tensor, rotations: Tensor, plane: Tensor, h: float) -> Tensor:
    return pts.new_empty((4, pts.shape[0], rotations.shape[0] * plane.shape[1]))


def _kpt_tv_bwd_impl(pts: Tensor, rotations: Tensor, plane: Tensor, grad_out: Tensor, h: float) -> list[Tensor]:
    _check_kernel_inputs("kplanes_tilted_tv_fuse_bwd", pts, rotations, plane, grad_out, taps=4)
    p = pts.contiguous()
    r = rotations.contiguous()
    c, hh, w = plane.shape[1:]
    b = p.shape[0]
    t = r.shape[0]
    stream = _stream(p.device)
    with _on_device(p.device):
        g = _channels_last(plane, stream)
        gout = grad_out.detach().to(dtype=torch.float32, device=p.device).contiguous()
        grad_pts = torch.zeros_like(p)
        grad_r = torch.zeros_like(r)
        grad_plane_cl = torch.zeros(g.shape, dtype=torch.float32, device=p.device)
        _core.kplanes_tilted_tv_fuse_grad_cuda(
            p.data_ptr(), r.data_ptr(), g.data_ptr(), gout.data_ptr(), grad_plane_cl.data_ptr(),
            grad_r.data_ptr(), grad_pts.data_ptr(), b, t, c, hh, w, float(h), stream,
        )
        grad_plane = _from_channels_last(grad_plane_cl, plane, stream)
    return [grad_pts, grad_r, grad_plane]


@torch.library.custom_op("quantem_cuda::kplanes_tilted_tv_fuse_bwd", mutates_args=())
def _kplanes_tilted_tv_fuse_bwd(
    pts: Tensor, rotations: Tensor, plane: Tensor, grad_out: Tensor, h: float
) -> list[Tensor]:
    return _kpt_tv_bwd_impl(pts, rotations, plane, grad_out, h)


@_kplanes_tilted_tv_fuse_bwd.register_fake
def _(pts: Tensor, rotations: Tensor, plane: Tensor, grad_out: Tensor, h: float) -> list[Tensor]:
    return [torch.empty_like(pts), torch.empty_like(rotations), torch.empty_like(plane)]


def _kpt_tv_setup_context(ctx, inputs, output) -> None:
    pts, rotations, plane, h = inputs
    ctx.save_for_backward(pts, rotations, plane)
    ctx.h = h


def _kpt_tv_backward(ctx, grad_out):
    pts, rotations, plane = ctx.saved_tensors
    grad_pts, grad_r, grad_plane = _kplanes_tilted_tv_fuse_bwd(pts, rotations, plane, grad_out, ctx.h)
    return grad_pts, grad_r, grad_plane, None


_kplanes_tilted_tv_fuse.register_autograd(_kpt_tv_backward, setup_context=_kpt_tv_setup_context)


class _KPlanesTiltedTV(torch.autograd.Function):
    """Eager counterpart of the registered four-tap op (see ``_KPlanesTilted``)."""

    @staticmethod
    def forward(ctx, pts: Tensor, rotations: Tensor, plane: Tensor, h: float) -> Tensor:
        ctx.save_for_backward(pts, rotations, plane)
        ctx.h = h
        return _kpt_tv_fwd_impl(pts, rotations, plane, h)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad_out):
        pts, rotations, plane = ctx.saved_tensors
        grad_pts, grad_r, grad_plane = _kpt_tv_bwd_impl(pts, rotations, plane, grad_out, ctx.h)
        return grad_pts, grad_r, grad_plane, None


# ── public wrapper ────────────────────────────────────────────────────────


def _validate(fn: str, pts: Tensor, rotations: Tensor, plane: Tensor) -> None:
    if pts.ndim != 2 or pts.shape[-1] != 3:
        raise ValueError(f"{fn} expects pts [B, 3], got {tuple(pts.shape)}")
    if rotations.ndim != 3 or rotations.shape[-2:] != (3, 3):
        raise ValueError(f"{fn} expects rotations [T, 3, 3], got {tuple(rotations.shape)}")
    if plane.ndim != 4 or plane.shape[0] != 3 * rotations.shape[0]:
        raise ValueError(
            f"{fn} expects plane [3*T, C, H, W] with T = "
            f"rotations.shape[0]; got plane {tuple(plane.shape)} for T={rotations.shape[0]}"
        )
    for name, t in (("pts", pts), ("rotations", rotations), ("plane", plane)):
        if t.dtype != torch.float32:
            raise TypeError(f"{fn} is fp32-only ({name} is {t.dtype}).")
        if not t.is_cuda:
            raise ValueError(f"{fn} requires CUDA tensors ({name} on {t.device}).")
    if plane.shape[1] * plane.shape[2] * plane.shape[3] >= 2**31:
        raise ValueError(
            f"{fn} uses 32-bit per-plane offsets; "
            f"C*H*W must be < 2^31, got plane {tuple(plane.shape)}"
        )


def kplanes_tilted_fuse(pts: Tensor, rotations: Tensor, plane: Tensor) -> Tensor:
    """Fused TILTED K-Planes feature interpolation for one multiscale level.

    For each point ``p`` and each rotation ``R_t``, bilinearly samples the
    three planes of rotation ``t`` at the (XY, ZX, YZ) pairs of ``R_t @ p``
    and Hadamard-multiplies them — equivalent to::

        rotated = torch.einsum("tij,bj->tbi", rotations, pts)
        coords = rotated[..., [[0, 1], [2, 0], [1, 2]]]      # (T, B, 3, 2)
        sampled = F.grid_sample(plane, coords.permute(0, 2, 1, 3).reshape(3*T, B, 1, 2),
                                align_corners=True, mode="bilinear",
                                padding_mode="border")
        out = sampled.squeeze(-1).view(T, 3, C, B).prod(1).permute(2, 0, 1).reshape(B, T*C)

    Differentiable w.r.t. all three inputs (analytic CUDA backward, with
    torch's border-clip zero-gradient convention for coordinates).

    Args:
        pts:       fp32 CUDA tensor ``[B, 3]``, coordinates in ``[-1, 1]``.
        rotations: fp32 CUDA tensor ``[T, 3, 3]``.
        plane:     fp32 CUDA tensor ``[3*T, C, H, W]`` (plane ``t*3 + p``).

    Returns:
        fp32 tensor ``[B, T*C]`` (``out[b, t*C + c]``), differentiable.
    """
    _validate("kplanes_tilted_fuse", pts, rotations, plane)
    if _eager(pts) and _eager(rotations) and _eager(plane):
        return _KPlanesTilted.apply(pts, rotations, plane)
    return _kplanes_tilted_fuse(pts, rotations, plane)


def kplanes_tilted_fuse_levels(pts: Tensor, rotations: Tensor, planes: list[Tensor]) -> list[Tensor]:
    """:func:`kplanes_tilted_fuse` for every level of a multiscale encoding in
    one launch per pass: ``planes[l]`` is level ``l``'s ``[3*T, C, H_l, W_l]``
    plane tensor (same ``T`` and ``C`` at every level, any resolution), and
    the result is the list of the levels' ``[B, T*C]`` features, each equal
    bit for bit to ``kplanes_tilted_fuse(pts, rotations, planes[l])``.
    Differentiable w.r.t. ``pts``, ``rotations`` and every plane tensor; the
    backward is one launch for all levels as well. At most 8 levels."""
    planes = list(planes)
    if not planes:
        raise ValueError("kplanes_tilted_fuse_levels expects at least one level")
    for plane in planes:
        _validate("kplanes_tilted_fuse_levels", pts, rotations, plane)
    if _eager(pts) and _eager(rotations) and all(_eager(pl) for pl in planes):
        return list(_KPlanesTiltedLevels.apply(pts, rotations, *planes))
    return _kplanes_tilted_fuse_levels(pts, rotations, planes)


def kplanes_tilted_tv_fuse(pts: Tensor, rotations: Tensor, plane: Tensor, h: float) -> Tensor:
    """Four-tap tilted K-Planes interpolation for finite-difference TV.

    For each point ``p`` and rotation ``R_t`` the ``kplanes_tilted_fuse``
    features at four locations:

        tap 0: R_t · p                 (bit-identical to kplanes_tilted_fuse)
        tap 1: R_t · p + h · R_t[:, 0]  (= R_t · (p + h·e_x))
        tap 2: R_t · p + h · R_t[:, 1]
        tap 3: R_t · p + h · R_t[:, 2]

    The rotation is evaluated once per (point, rotation) and the column
    offsets once per rotation.

    Args:
        pts:       fp32 CUDA tensor ``[B, 3]``.
        rotations: fp32 CUDA tensor ``[T, 3, 3]``.
        plane:     fp32 CUDA tensor ``[3*T, C, H, W]``.
        h:         finite-difference step in the ``[-1, 1]`` coordinates (no gradient).

    Returns:
        fp32 tensor ``[4, B, T*C]``, tap outermost, differentiable w.r.t.
        pts, rotations and plane.
    """
    _validate("kplanes_tilted_tv_fuse", pts, rotations, plane)
    if _eager(pts) and _eager(rotations) and _eager(plane):
        return _KPlanesTiltedTV.apply(pts, rotations, plane, float(h))
    return _kplanes_tilted_tv_fuse(pts, rotations, plane, float(h))
