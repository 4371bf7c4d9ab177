"""torch registration of the 3-D total-variation kernels.

Mirrors the reference's src/quantem/cuda/core/_ops.py (same op names, schemas,
fake implementations, autograd wiring, public wrappers and error messages):

    quantem_cuda::tv_loss_iso_3d(Tensor volume, float eps) -> Tensor        (:39-50)
    quantem_cuda::tv_loss_iso_3d_bwd(Tensor volume, Tensor grad_out, float eps) -> Tensor
    quantem_cuda::tv_loss_sq_3d(Tensor volume) -> Tensor                    (:98-109)
    quantem_cuda::tv_loss_sq_3d_bwd(Tensor volume, Tensor grad_out) -> Tensor
    quantem_cuda::tv_loss_l1_3d(Tensor volume) -> Tensor (3,)               (:187-198)
    quantem_cuda::tv_loss_l1_3d_bwd(Tensor volume, Tensor grad_out) -> Tensor

and adds single-sweep forward + gradient ops that read the volume once and
write the loss and the gradient together (8 B/voxel of HBM traffic instead of
the 12 B/voxel of the forward/backward pair):

    quantem_cuda::tv_loss_{iso,sq,l1}_3d_fwd_grad(volume, grad_out[, eps]) -> (loss, grad)

Differences in mechanism (results are the same): the losses are reduced
deterministically in the kernel (fixed-order fp64 partial sums) instead of
with fp32 atomics, the isotropic 1/N is folded into the kernel, and the
gradient buffers are fully written by the kernel (``empty_like`` instead of
``zeros_like``).
"""

from __future__ import annotations

import torch
from torch import Tensor

from quantem.cuda import _core
from quantem.cuda._common import _as_batched, _launch_args, _workspace

_SQ, _ISO, _L1 = _core.TV_SQ, _core.TV_ISO, _core.TV_L1
_LOSS, _GRAD, _OVERWRITE = _core.TV_LOSS, _core.TV_GRAD, _core.TV_ACC_OVERWRITE


def _iso_n_corners(shape: tuple[int, ...]) -> int:
    b, d, h, w = shape
    return max(1, b * (d - 1) * (h - 1) * (w - 1))


def _run(
    variant: int,
    flags: int,
    vol: Tensor,
    g: Tensor | None,
    acc: Tensor | None,
    grad: Tensor | None,
    eps: float,
    scale: float,
    stream: int,
) -> None:
    b, d, h, w = vol.shape
    ws = _workspace(vol.device) if flags & _LOSS else None
    with _on_device(vol.device):
        _core.tv_loss_3d_slab_cuda(
            variant,
            flags,
            vol.data_ptr(),
            0 if g is None else g.data_ptr(),
            0 if acc is None else acc.data_ptr(),
            0 if grad is None else grad.data_ptr(),
            b,
            d,
            h,
            w,
            0,
            d,
            0,
            0,
            float(eps),
            float(scale),
            0 if ws is None else ws.data_ptr(),
            0 if ws is None else ws.numel(),
            stream,
        )


class _NoContext:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NO_CONTEXT = _NoContext()


def _on_device(device: torch.device):
    """torch.cuda.device(device), or nothing when it is already current (the
    context manager costs host time on every call)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return _NO_CONTEXT
    return torch.cuda.device(device)


def _eager(x: Tensor) -> bool:
    """True for a plain tensor outside torch.compile: the public wrappers of
    the single-sweep ops then call their implementation directly instead of
    through the torch.library dispatcher, whose Python-side cost per call
    (about 60 us) is comparable to a sweep's device time on small volumes.
    Under compilation, and for tensor subclasses (fake tensors), the
    registered op is used."""
    return type(x) is torch.Tensor and not torch.compiler.is_compiling()


def _upstream(grad_out: Tensor | float, n: int, device: torch.device) -> Tensor:
    if (isinstance(grad_out, Tensor) and grad_out.dtype == torch.float32 and grad_out.device == device
            and grad_out.numel() == n and grad_out.is_contiguous()):
        return grad_out.detach().view(n)
    if isinstance(grad_out, Tensor):
        return grad_out.detach().to(dtype=torch.float32, device=device).reshape(n).contiguous()
    return torch.full((n,), float(grad_out), dtype=torch.float32, device=device)


# ── isotropic 3-D TV ──────────────────────────────────────────────────────


def _iso_fwd_impl(volume: Tensor, eps: float) -> Tensor:
    vol, b, d, h, w, stream = _launch_args(volume)
    acc = torch.empty(1, dtype=torch.float32, device=vol.device)
    scale = 1.0 / float(_iso_n_corners(vol.shape))
    _run(_ISO, _LOSS | _OVERWRITE, vol, None, acc, None, eps, scale, stream)
    return acc.squeeze(0)


@torch.library.custom_op("quantem_cuda::tv_loss_iso_3d", mutates_args=())
def _tv_loss_iso_3d(volume: Tensor, eps: float) -> Tensor:
    return _iso_fwd_impl(volume, eps)


@_tv_loss_iso_3d.register_fake
def _(volume: Tensor, eps: float) -> Tensor:
    return volume.new_empty(())


def _iso_bwd_impl(volume: Tensor, grad_out: Tensor, eps: float) -> Tensor:
    vol, b, d, h, w, stream = _launch_args(volume)
    g = _upstream(grad_out, 1, vol.device)
    grad_vol = torch.empty_like(vol)
    scale = 1.0 / float(_iso_n_corners(vol.shape))
    _run(_ISO, _GRAD, vol, g, None, grad_vol, eps, scale, stream)
    return grad_vol


@torch.library.custom_op("quantem_cuda::tv_loss_iso_3d_bwd", mutates_args=())
def _tv_loss_iso_3d_bwd(volume: Tensor, grad_out: Tensor, eps: float) -> Tensor:
    return _iso_bwd_impl(volume, grad_out, eps)


@_tv_loss_iso_3d_bwd.register_fake
def _(volume: Tensor, grad_out: Tensor, eps: float) -> Tensor:
    return torch.empty_like(volume)


def _iso_setup_context(ctx, inputs, output) -> None:
    volume, eps = inputs
    ctx.save_for_backward(volume)
    ctx.eps = eps


def _iso_backward(ctx, grad_out):
    (volume,) = ctx.saved_tensors
    return _tv_loss_iso_3d_bwd(volume, grad_out, ctx.eps), None


_tv_loss_iso_3d.register_autograd(_iso_backward, setup_context=_iso_setup_context)


# ── squared-anisotropic 3-D TV (quantem tv_vol parity) ────────────────────


def _sq_fwd_impl(volume: Tensor) -> Tensor:
    vol, b, d, h, w, stream = _launch_args(volume)
    acc = torch.empty(1, dtype=torch.float32, device=vol.device)
    _run(_SQ, _LOSS | _OVERWRITE, vol, None, acc, None, 0.0, 1.0, stream)
    return acc.squeeze(0)


@torch.library.custom_op("quantem_cuda::tv_loss_sq_3d", mutates_args=())
def _tv_loss_sq_3d(volume: Tensor) -> Tensor:
    return _sq_fwd_impl(volume)


@_tv_loss_sq_3d.register_fake
def _(volume: Tensor) -> Tensor:
    return volume.new_empty(())


def _sq_bwd_impl(volume: Tensor, grad_out: Tensor) -> Tensor:
    vol, b, d, h, w, stream = _launch_args(volume)
    g = _upstream(grad_out, 1, vol.device)
    grad_vol = torch.empty_like(vol)
    _run(_SQ, _GRAD, vol, g, None, grad_vol, 0.0, 1.0, stream)
    return grad_vol


@torch.library.custom_op("quantem_cuda::tv_loss_sq_3d_bwd", mutates_args=())
def _tv_loss_sq_3d_bwd(volume: Tensor, grad_out: Tensor) -> Tensor:
    return _sq_bwd_impl(volume, grad_out)


@_tv_loss_sq_3d_bwd.register_fake
def _(volume: Tensor, grad_out: Tensor) -> Tensor:
    return torch.empty_like(volume)


def _sq_setup_context(ctx, inputs, output) -> None:
    (volume,) = inputs
    ctx.save_for_backward(volume)


def _sq_backward(ctx, grad_out):
    (volume,) = ctx.saved_tensors
    return _tv_loss_sq_3d_bwd(volume, grad_out)


_tv_loss_sq_3d.register_autograd(_sq_backward, setup_context=_sq_setup_context)


# ── L1-anisotropic 3-D TV (per-axis sums) ─────────────────────────────────


def _l1_fwd_impl(volume: Tensor) -> Tensor:
    vol, b, d, h, w, stream = _launch_args(volume)
    acc = torch.empty(3, dtype=torch.float32, device=vol.device)
    _run(_L1, _LOSS | _OVERWRITE, vol, None, acc, None, 0.0, 1.0, stream)
    return acc


@torch.library.custom_op("quantem_cuda::tv_loss_l1_3d", mutates_args=())
def _tv_loss_l1_3d(volume: Tensor) -> Tensor:
    return _l1_fwd_impl(volume)


@_tv_loss_l1_3d.register_fake
def _(volume: Tensor) -> Tensor:
    return volume.new_empty((3,))


def _l1_bwd_impl(volume: Tensor, grad_out: Tensor) -> Tensor:
    vol, b, d, h, w, stream = _launch_args(volume)
    g = _upstream(grad_out, 3, vol.device)
    grad_vol = torch.empty_like(vol)
    _run(_L1, _GRAD, vol, g, None, grad_vol, 0.0, 1.0, stream)
    return grad_vol


@torch.library.custom_op("quantem_cuda::tv_loss_l1_3d_bwd", mutates_args=())
def _tv_loss_l1_3d_bwd(volume: Tensor, grad_out: Tensor) -> Tensor:
    return _l1_bwd_impl(volume, grad_out)


@_tv_loss_l1_3d_bwd.register_fake
def _(volume: Tensor, grad_out: Tensor) -> Tensor:
    return torch.empty_like(volume)


def _l1_setup_context(ctx, inputs, output) -> None:
    (volume,) = inputs
    ctx.save_for_backward(volume)


def _l1_backward(ctx, grad_out):
    (volume,) = ctx.saved_tensors
    return _tv_loss_l1_3d_bwd(volume, grad_out)


_tv_loss_l1_3d.register_autograd(_l1_backward, setup_context=_l1_setup_context)


# ── single-sweep forward + gradient ───────────────────────────────────────


def _iso_fwd_grad_impl(volume: Tensor, grad_out: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    vol, b, d, h, w, stream = _launch_args(volume)
    g = _upstream(grad_out, 1, vol.device)
    acc = torch.empty(1, dtype=torch.float32, device=vol.device)
    grad_vol = torch.empty_like(vol)
    scale = 1.0 / float(_iso_n_corners(vol.shape))
    _run(_ISO, _LOSS | _GRAD | _OVERWRITE, vol, g, acc, grad_vol, eps, scale, stream)
    return acc.squeeze(0), grad_vol


@torch.library.custom_op("quantem_cuda::tv_loss_iso_3d_fwd_grad", mutates_args=())
def _tv_loss_iso_3d_fwd_grad(volume: Tensor, grad_out: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    return _iso_fwd_grad_impl(volume, grad_out, eps)


@_tv_loss_iso_3d_fwd_grad.register_fake
def _(volume: Tensor, grad_out: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    return volume.new_empty(()), torch.empty_like(volume)


def _sq_fwd_grad_impl(volume: Tensor, grad_out: Tensor) -> tuple[Tensor, Tensor]:
    vol, b, d, h, w, stream = _launch_args(volume)
    g = _upstream(grad_out, 1, vol.device)
    acc = torch.empty(1, dtype=torch.float32, device=vol.device)
    grad_vol = torch.empty_like(vol)
    _run(_SQ, _LOSS | _GRAD | _OVERWRITE, vol, g, acc, grad_vol, 0.0, 1.0, stream)
    return acc.squeeze(0), grad_vol


@torch.library.custom_op("quantem_cuda::tv_loss_sq_3d_fwd_grad", mutates_args=())
def _tv_loss_sq_3d_fwd_grad(volume: Tensor, grad_out: Tensor) -> tuple[Tensor, Tensor]:
    return _sq_fwd_grad_impl(volume, grad_out)


@_tv_loss_sq_3d_fwd_grad.register_fake
def _(volume: Tensor, grad_out: Tensor) -> tuple[Tensor, Tensor]:
    return volume.new_empty(()), torch.empty_like(volume)


def _l1_fwd_grad_impl(volume: Tensor, grad_out: Tensor) -> tuple[Tensor, Tensor]:
    vol, b, d, h, w, stream = _launch_args(volume)
    g = _upstream(grad_out, 3, vol.device)
    acc = torch.empty(3, dtype=torch.float32, device=vol.device)
    grad_vol = torch.empty_like(vol)
    _run(_L1, _LOSS | _GRAD | _OVERWRITE, vol, g, acc, grad_vol, 0.0, 1.0, stream)
    return acc, grad_vol


@torch.library.custom_op("quantem_cuda::tv_loss_l1_3d_fwd_grad", mutates_args=())
def _tv_loss_l1_3d_fwd_grad(volume: Tensor, grad_out: Tensor) -> tuple[Tensor, Tensor]:
    return _l1_fwd_grad_impl(volume, grad_out)


@_tv_loss_l1_3d_fwd_grad.register_fake
def _(volume: Tensor, grad_out: Tensor) -> tuple[Tensor, Tensor]:
    return volume.new_empty((3,)), torch.empty_like(volume)


# ── several terms in one sweep ────────────────────────────────────────────

_TERM_SQ, _TERM_ISO, _TERM_L1 = _core.TV_TERM_SQ, _core.TV_TERM_ISO, _core.TV_TERM_L1


def _multi_fwd_grad_impl(volume: Tensor, weights: Tensor, terms: int, eps: float) -> tuple[Tensor, Tensor]:
    """weights = [w_sq, w_iso, w_d, w_h, w_w]; returns ([sq sum, iso mean, l1_d,
    l1_h, l1_w], Σ_term w·∂term/∂volume) for the terms in the bit mask."""
    vol, b, d, h, w, stream = _launch_args(volume)
    n = float(_iso_n_corners(vol.shape))
    g = weights.detach().to(dtype=torch.float32, device=vol.device).reshape(5).contiguous()
    acc = torch.empty(5, dtype=torch.float32, device=vol.device)
    grad_vol = torch.empty_like(vol)
    ws = _workspace(vol.device)
    with _on_device(vol.device):
        _core.tv_loss_mix_3d_fwd_grad_cuda(
            int(terms), _OVERWRITE, vol.data_ptr(), g.data_ptr(), acc.data_ptr(), grad_vol.data_ptr(),
            b, d, h, w, float(eps), 1.0 / n, ws.data_ptr(), ws.numel(), stream,
        )
    return acc, grad_vol


@torch.library.custom_op("quantem_cuda::tv_loss_multi_3d_fwd_grad", mutates_args=())
def _tv_loss_multi_3d_fwd_grad(volume: Tensor, weights: Tensor, terms: int, eps: float) -> tuple[Tensor, Tensor]:
    return _multi_fwd_grad_impl(volume, weights, terms, eps)


@_tv_loss_multi_3d_fwd_grad.register_fake
def _(volume: Tensor, weights: Tensor, terms: int, eps: float) -> tuple[Tensor, Tensor]:
    return volume.new_empty((5,)), torch.empty_like(volume)


# ── eager autograd ────────────────────────────────────────────────────────
#
# The same implementations under torch.autograd.Function, used by the public
# wrappers for plain tensors outside torch.compile: the registered ops above
# stay what torch.compile and torch.ops.quantem_cuda.* see, while an eager
# call skips the torch.library dispatcher's host cost. Backward is
# once-differentiable, as the registered ops' backward is not differentiable
# either.


class _IsoTV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, volume: Tensor, eps: float) -> Tensor:
        ctx.save_for_backward(volume)
        ctx.eps = eps
        return _iso_fwd_impl(volume, eps)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad_out):
        (volume,) = ctx.saved_tensors
        return _iso_bwd_impl(volume, grad_out, ctx.eps), None


class _SqTV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, volume: Tensor) -> Tensor:
        ctx.save_for_backward(volume)
        return _sq_fwd_impl(volume)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad_out):
        (volume,) = ctx.saved_tensors
        return _sq_bwd_impl(volume, grad_out)


class _L1TV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, volume: Tensor) -> Tensor:
        ctx.save_for_backward(volume)
        return _l1_fwd_impl(volume)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad_out):
        (volume,) = ctx.saved_tensors
        return _l1_bwd_impl(volume, grad_out)


# ── public wrappers ───────────────────────────────────────────────────────


def tv_loss_iso_3d(volume: Tensor, eps: float = 1e-8) -> Tensor:
    """Isotropic 3-D total-variation loss (fused CUDA forward + backward).

        loss = mean over corners of sqrt( dd² + dh² + dw² + eps )

    where dd/dh/dw are forward differences along the three trailing dims
    and the corner set is ``[0, D−2] × [0, H−2] × [0, W−2]`` per leading
    slice. Leading dims (channels and/or batch) are flattened and included
    in the mean.

    Args:
        volume: fp32 CUDA tensor, shape ``[D, H, W]`` or ``[..., D, H, W]``.
        eps:    smoothing constant inside the sqrt (default 1e-8).

    Returns:
        0-dim fp32 tensor on the same device as ``volume``; differentiable.
    """
    vol = _as_batched(volume, "tv_loss_iso_3d")
    return _IsoTV.apply(vol, float(eps)) if _eager(vol) else _tv_loss_iso_3d(vol, eps)


def tv_loss_sq_3d(volume: Tensor) -> Tensor:
    """Squared-anisotropic 3-D total-variation sum (fused CUDA kernels).

        loss = Σ (Δd)² + Σ (Δh)² + Σ (Δw)²

    over forward differences along the three trailing dims, each summed over
    its full complementary index range — quantem's ``tv_vol`` regularizer
    before its ``weight / numel`` scaling. Leading dims are flattened and
    included in the sum.

    Args:
        volume: fp32 CUDA tensor, shape ``[D, H, W]`` or ``[..., D, H, W]``.

    Returns:
        0-dim fp32 tensor on the same device as ``volume``; differentiable.
    """
    vol = _as_batched(volume, "tv_loss_sq_3d")
    return _SqTV.apply(vol) if _eager(vol) else _tv_loss_sq_3d(vol)


def tv_loss_l1_3d(volume: Tensor) -> Tensor:
    """Per-axis L1-anisotropic 3-D total-variation sums (fused CUDA kernels).

        sums = [ Σ|Δd|, Σ|Δh|, Σ|Δw| ]

    over forward differences along the three trailing dims, each summed over
    its full complementary index range. The sums are raw; quantem's
    ptychography ``_calc_tv_loss(array, (w_z, w_xy))`` on ``[S, H, W]`` is
    ``(w_z·sums[0]/((S-1)HW) + w_xy·sums[1]/(S(H-1)W) + w_xy·sums[2]/(SH(W-1)))
    / n_active_axes`` (see :func:`ptycho_tv_loss`). A trailing dim of size 1
    contributes an empty sum of 0; the gradient uses ``sign(0) = 0``.

    Args:
        volume: fp32 CUDA tensor, shape ``[D, H, W]`` or ``[..., D, H, W]``.

    Returns:
        Shape-``(3,)`` fp32 tensor on the same device; differentiable.
    """
    vol = _as_batched(volume, "tv_loss_l1_3d")
    return _L1TV.apply(vol) if _eager(vol) else _tv_loss_l1_3d(vol)


def tv_loss_iso_3d_fwd_grad(
    volume: Tensor, grad_out: Tensor | float = 1.0, eps: float = 1e-8
) -> tuple[Tensor, Tensor]:
    """Isotropic TV loss and ``grad_out · ∂loss/∂volume`` in one HBM sweep.

    Returns ``(loss, grad)`` with ``loss`` equal to :func:`tv_loss_iso_3d` and
    ``grad`` shaped like ``volume``. Not differentiable itself.
    """
    vol = _as_batched(volume, "tv_loss_iso_3d_fwd_grad")
    op = _iso_fwd_grad_impl if _eager(vol) else _tv_loss_iso_3d_fwd_grad
    loss, grad = op(vol, _upstream(grad_out, 1, vol.device), float(eps))
    return loss, grad.view(volume.shape)


def tv_loss_sq_3d_fwd_grad(volume: Tensor, grad_out: Tensor | float = 1.0) -> tuple[Tensor, Tensor]:
    """Squared TV sum and ``grad_out · ∂sum/∂volume`` in one HBM sweep."""
    vol = _as_batched(volume, "tv_loss_sq_3d_fwd_grad")
    op = _sq_fwd_grad_impl if _eager(vol) else _tv_loss_sq_3d_fwd_grad
    loss, grad = op(vol, _upstream(grad_out, 1, vol.device))
    return loss, grad.view(volume.shape)


def tv_loss_l1_3d_fwd_grad(
    volume: Tensor, grad_out: Tensor | float | tuple[float, float, float] = 1.0
) -> tuple[Tensor, Tensor]:
    """Per-axis L1 TV sums and ``Σ_axis grad_out[axis] · ∂sums[axis]/∂volume``
    in one HBM sweep. ``grad_out`` is a 3-vector (or a scalar for all axes)."""
    vol = _as_batched(volume, "tv_loss_l1_3d_fwd_grad")
    if isinstance(grad_out, (tuple, list)):
        g = _host_values(grad_out, vol.device)
    elif isinstance(grad_out, Tensor):
        g = grad_out.detach().to(dtype=torch.float32, device=vol.device)
        g = g.expand(3) if g.numel() == 1 else g.reshape(3)
    else:
        g = float(grad_out)
    g = _upstream(g, 3, vol.device)
    op = _l1_fwd_grad_impl if _eager(vol) else _tv_loss_l1_3d_fwd_grad
    sums, grad = op(vol, g)
    return sums, grad.view(volume.shape)


def _weight(x, n: int, device) -> Tensor:
    if isinstance(x, Tensor):
        t = x.detach().to(dtype=torch.float32, device=device).reshape(-1)
        return t.expand(n) if t.numel() == 1 else t.reshape(n)
    if isinstance(x, (tuple, list)):
        if len(x) != n:
            raise ValueError(f"expected {n} weights, got {len(x)}")
        return _host_values(x, device)
    return torch.full((n,), float(x), dtype=torch.float32, device=device)


def _host_values(values, device) -> Tensor:
    """A few host floats on the device through pinned memory: the copy is
    queued on the current stream without waiting for it (a copy from pageable
    memory would first synchronise with the stream)."""
    host = torch.tensor([float(v) for v in values], dtype=torch.float32).pin_memory()
    return host.to(device, non_blocking=True)


def tv_loss_multi_3d_fwd_grad(
    volume: Tensor,
    *,
    sq: Tensor | float | None = None,
    iso: Tensor | float | None = None,
    l1: Tensor | float | tuple[float, float, float] | None = None,
    eps: float = 1e-8,
) -> tuple[dict[str, Tensor], Tensor]:
    """Several TV terms of one volume and the gradient of their weighted sum,
    reading the volume once.

    ``sq`` and ``iso`` weight :func:`tv_loss_sq_3d` and :func:`tv_loss_iso_3d`
    (the mean over corners, ``eps`` inside the square root); ``l1`` weights
    the three per-axis sums of :func:`tv_loss_l1_3d` (one value for all axes
    or three). A term left as ``None`` is not computed. Returns
    ``(losses, grad)``: ``losses`` maps "sq", "iso", "l1" (for the terms
    given) to what the single-term ops return, and ``grad`` is
    ``Σ weight · ∂term/∂volume``. With two or three terms one sweep computes
    everything (8 B of HBM traffic per voxel instead of 8 B per term); with
    one term this is that term's single sweep. Not differentiable itself.
    """
    vol = _as_batched(volume, "tv_loss_multi_3d_fwd_grad")
    dev = vol.device
    terms = (_TERM_SQ if sq is not None else 0) | (_TERM_ISO if iso is not None else 0) | (
        _TERM_L1 if l1 is not None else 0)
    if terms == 0:
        raise ValueError("tv_loss_multi_3d_fwd_grad needs at least one of sq, iso, l1")
    if terms in (_TERM_SQ, _TERM_ISO, _TERM_L1):
        eager = _eager(vol)
        if terms == _TERM_SQ:
            op = _sq_fwd_grad_impl if eager else _tv_loss_sq_3d_fwd_grad
            loss, grad = op(vol, _weight(sq, 1, dev))
            return {"sq": loss}, grad.view(volume.shape)
        if terms == _TERM_ISO:
            op = _iso_fwd_grad_impl if eager else _tv_loss_iso_3d_fwd_grad
            loss, grad = op(vol, _weight(iso, 1, dev), float(eps))
            return {"iso": loss}, grad.view(volume.shape)
        op = _l1_fwd_grad_impl if eager else _tv_loss_l1_3d_fwd_grad
        sums, grad = op(vol, _weight(l1, 3, dev))
        return {"l1": sums}, grad.view(volume.shape)
    zero1 = torch.zeros(1, dtype=torch.float32, device=dev)
    weights = torch.cat([
        _weight(sq, 1, dev) if sq is not None else zero1,
        _weight(iso, 1, dev) if iso is not None else zero1,
        _weight(l1, 3, dev) if l1 is not None else zero1.expand(3),
    ])
    op = _multi_fwd_grad_impl if _eager(vol) else _tv_loss_multi_3d_fwd_grad
    acc, grad = op(vol, weights, terms, float(eps))
    losses = {}
    if sq is not None:
        losses["sq"] = acc[0]
    if iso is not None:
        losses["iso"] = acc[1]
    if l1 is not None:
        losses["l1"] = acc[2:5]
    return losses, grad.view(volume.shape)


def ptycho_tv_loss(array: Tensor, weight: tuple[float, float]) -> Tensor:
    """quantem's ptychography ``ObjectConstraints._calc_tv_loss(array, weight)``
    on a ``[S, H, W]`` array, built on :func:`tv_loss_l1_3d` (the recipe the
    reference documents in core/_ops.py:239-247 and tests at
    test_tv_loss.py:213-235): per-axis means weighted ``(w_z, w_xy, w_xy)``,
    divided by the number of axes with a positive weight."""
    if array.ndim != 3:
        raise ValueError(f"ptycho_tv_loss expects [S, H, W], got shape {tuple(array.shape)}")
    s, h, w = array.shape
    sums = tv_loss_l1_3d(array)
    counts = sums.new_tensor([(s - 1) * h * w, s * (h - 1) * w, s * h * (w - 1)]).clamp(min=1)
    wz, wxy = float(weight[0]), float(weight[1])
    wt = sums.new_tensor([wz, wxy, wxy])
    active = max(1, int(wz > 0) + 2 * int(wxy > 0))
    return (wt * sums / counts).sum() / active


def tv_vol_loss(volume: Tensor, weight: float) -> Tensor:
    """quantem's ``tv_vol`` volume regulariser: ``weight`` times the squared
    anisotropic TV sum of :func:`tv_loss_sq_3d` divided by the number of
    voxels (the scaling the reference's docstring names, core/_ops.py:170-172).
    A zero weight returns an exact zero that still carries a (zero) gradient."""
    loss = tv_loss_sq_3d(volume)
    return loss * (float(weight) / max(1, volume.numel()))
