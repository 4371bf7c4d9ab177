"""Helpers shared by the op layers (mirrors the reference's
src/quantem/cuda/_common.py:11-33, same validation messages)."""

from __future__ import annotations

import torch
from torch import Tensor

from quantem.cuda import _core


def _launch_args(volume: Tensor) -> tuple[Tensor, int, int, int, int, int]:
    vol = volume.contiguous()
    b, d, h, w = vol.shape
    stream = torch.cuda.current_stream(vol.device).cuda_stream
    return vol, b, d, h, w, stream


def _as_batched(volume: Tensor, fn: str) -> Tensor:
    if volume.ndim < 3:
        raise ValueError(
            f"{fn} expects [..., D, H, W] with ndim >= 3, got shape {tuple(volume.shape)}"
        )
    if volume.dtype != torch.float32:
        raise TypeError(f"{fn} is fp32-only (got {volume.dtype}).")
    if not volume.is_cuda:
        raise ValueError(f"{fn} requires a CUDA tensor (got device {volume.device}).")
    d, h, w = volume.shape[-3:]
    return volume.reshape(-1, d, h, w)


def _workspace(device: torch.device) -> Tensor:
    """Scratch for the deterministic two-pass TV reductions (per-CTA partial
    sums). Allocated from torch's caching allocator for every call, so calls on
    different streams never share one."""
    nbytes = int(_core.tv_loss_3d_workspace_bytes(0, 0, 0, 0))
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def cudart_version() -> int:
    """CUDA runtime version the extension was compiled against (e.g. 12090)."""
    return int(_core.__cudart_version__)
