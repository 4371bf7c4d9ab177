"""Pure-torch CPU definitions of the hot path (TEST AND BASELINE INFRASTRUCTURE).

The reference pins its kernels against torch expressions in its test files:
the TV losses at tests/core/test_tv_loss.py:13-27 (isotropic, squared) and
:144-153 (L1), the tilted K-Planes level at
tests/core/ml/test_kplanes_tilted.py:26-40 (rotation, then grid_sample of the
three plane projections with align_corners=True and border padding, product
over the planes). This module states the same definitions with torch
operations, so that their CPU cost can be timed next to the C oracle
(``bench.py``'s CPU baselines) with autograd supplying the gradients, as the
reference's tests do. Nothing in the product imports it.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor


def _batched(volume: Tensor) -> Tensor:
    return volume.reshape(-1, *volume.shape[-3:])


def _forward_diffs(v: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """Forward differences of a [B, D, H, W] volume along D, H and W."""
    return v[:, 1:] - v[:, :-1], v[:, :, 1:] - v[:, :, :-1], v[:, :, :, 1:] - v[:, :, :, :-1]


def tv_iso(volume: Tensor, eps: float) -> Tensor:
    """Mean over the corners [0, D-2] x [0, H-2] x [0, W-2] of
    sqrt(dd^2 + dh^2 + dw^2 + eps)."""
    dd, dh, dw = _forward_diffs(_batched(volume))
    s = dd[:, :, :-1, :-1] ** 2 + dh[:, :-1, :, :-1] ** 2 + dw[:, :-1, :-1, :] ** 2 + eps
    return s.sqrt().mean()


def tv_sq(volume: Tensor) -> Tensor:
    """Sum over the three axes of the squared forward differences, each over
    its full range."""
    return sum((d * d).sum() for d in _forward_diffs(_batched(volume)))


def tv_l1(volume: Tensor) -> Tensor:
    """Per-axis sums of |forward difference|, shape (3,), order (D, H, W)."""
    return torch.stack([d.abs().sum() for d in _forward_diffs(_batched(volume))])


# plane p of rotation t samples the rotated point's coordinate pair
# (x, y) for XY, (z, x) for ZX, (y, z) for YZ; the first goes along W
_PAIRS = ((0, 1), (2, 0), (1, 2))


def kplanes_tilted(pts: Tensor, rotations: Tensor, plane: Tensor) -> Tensor:
    """out[b, t*C + c] = prod_p bilinear(plane[3t + p], pair_p(R_t pts_b)),
    [N, T*C]."""
    T, N, C = rotations.shape[0], pts.shape[0], plane.shape[1]
    rotated = torch.matmul(pts, rotations.transpose(1, 2))  # [T, N, 3]
    grids = torch.stack([rotated[..., list(pair)] for pair in _PAIRS], dim=1)  # [T, 3, N, 2]
    sampled = F.grid_sample(plane, grids.reshape(3 * T, N, 1, 2), mode="bilinear", padding_mode="border",
                            align_corners=True)  # [3T, C, N, 1]
    per_plane = sampled.reshape(T, 3, C, N)
    return (per_plane[:, 0] * per_plane[:, 1] * per_plane[:, 2]).permute(2, 0, 1).reshape(N, T * C)
