"""Shared kernels usable across quantem modules: 3-D total-variation losses.

``quantem.cuda.core.ml`` holds the K-Planes kernels (quantem.core.ml).
Mirrors the reference's src/quantem/cuda/core/__init__.py.
"""

from quantem.cuda.core import ml as ml
from quantem.cuda.core._ops import (
    ptycho_tv_loss as ptycho_tv_loss,
    tv_loss_iso_3d as tv_loss_iso_3d,
    tv_loss_iso_3d_fwd_grad as tv_loss_iso_3d_fwd_grad,
    tv_loss_l1_3d as tv_loss_l1_3d,
    tv_loss_l1_3d_fwd_grad as tv_loss_l1_3d_fwd_grad,
    tv_loss_multi_3d_fwd_grad as tv_loss_multi_3d_fwd_grad,
    tv_loss_sq_3d as tv_loss_sq_3d,
    tv_loss_sq_3d_fwd_grad as tv_loss_sq_3d_fwd_grad,
    tv_vol_loss as tv_vol_loss,
)
