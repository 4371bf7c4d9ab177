"""Input validation of the public wrappers, on CPU tensors (mirrors the
reference's CPU-tier tests: test_tv_loss.py:125-138, 264-266;
test_kplanes_tilted.py:168-186)."""

from __future__ import annotations

import pytest
import torch

from quantem.cuda.core import (
    ptycho_tv_loss,
    tv_loss_iso_3d,
    tv_loss_iso_3d_fwd_grad,
    tv_loss_l1_3d,
    tv_loss_l1_3d_fwd_grad,
    tv_loss_sq_3d,
    tv_loss_sq_3d_fwd_grad,
)
from quantem.cuda.core.ml import kplanes_tilted_fuse


def test_rejects_cpu_tensor():
    vol = torch.rand(8, 8, 8)
    for fn in (tv_loss_iso_3d, tv_loss_sq_3d, tv_loss_l1_3d):
        with pytest.raises(ValueError, match="CUDA"):
            fn(vol)
    for fn in (tv_loss_iso_3d_fwd_grad, tv_loss_sq_3d_fwd_grad, tv_loss_l1_3d_fwd_grad):
        with pytest.raises(ValueError, match="CUDA"):
            fn(vol)


def test_rejects_bad_dtype_and_ndim():
    with pytest.raises(TypeError, match="fp32"):
        tv_loss_iso_3d(torch.rand(8, 8, 8, dtype=torch.float64))
    with pytest.raises(ValueError, match="ndim"):
        tv_loss_sq_3d(torch.rand(8, 8))
    with pytest.raises(ValueError, match="ndim"):
        tv_loss_l1_3d(torch.rand(8))
    with pytest.raises(ValueError, match=r"\[S, H, W\]"):
        ptycho_tv_loss(torch.rand(2, 3, 4, 5), (1.0, 1.0))


def test_kplanes_cpu_rejected():
    pts = torch.rand(8, 3)
    rotations = torch.rand(2, 3, 3)
    plane = torch.rand(6, 4, 9, 9)
    with pytest.raises(ValueError, match="CUDA"):
        kplanes_tilted_fuse(pts, rotations, plane)


def test_kplanes_tv_cpu_rejected_and_messages():
    from quantem.cuda.core.ml import kplanes_tilted_tv_fuse

    pts = torch.rand(8, 3)
    rotations = torch.rand(2, 3, 3)
    plane = torch.rand(6, 4, 9, 9)
    with pytest.raises(ValueError, match="CUDA"):
        kplanes_tilted_tv_fuse(pts, rotations, plane, h=0.01)
    with pytest.raises(ValueError, match=r"kplanes_tilted_tv_fuse expects pts \[B, 3\]"):
        kplanes_tilted_tv_fuse(pts[:, :2], rotations, plane, h=0.01)
    with pytest.raises(ValueError, match=r"3\*T"):
        kplanes_tilted_tv_fuse(pts, rotations, plane[:3], h=0.01)
    with pytest.raises(TypeError, match="kplanes_tilted_tv_fuse is fp32-only"):
        kplanes_tilted_tv_fuse(pts.double(), rotations, plane, h=0.01)


def test_kplanes_tv_fake_shapes():
    from quantem.cuda.core.ml import _ops  # noqa: F401  (registers the ops)
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        p = torch.empty(10, 3, device="cuda")
        r = torch.empty(2, 3, 3, device="cuda")
        g = torch.empty(6, 8, 5, 5, device="cuda")
        out = torch.ops.quantem_cuda.kplanes_tilted_tv_fuse(p, r, g, 0.1)
        assert tuple(out.shape) == (4, 10, 16)
        gp, gr, gg = torch.ops.quantem_cuda.kplanes_tilted_tv_fuse_bwd(p, r, g, out, 0.1)
        assert tuple(gp.shape) == (10, 3) and tuple(gr.shape) == (2, 3, 3) and tuple(gg.shape) == (6, 8, 5, 5)


def test_kplanes_shape_validation_messages():
    pts = torch.rand(16, 3)
    rotations = torch.rand(2, 3, 3)
    plane = torch.rand(6, 4, 9, 9)
    with pytest.raises(ValueError, match=r"pts \[B, 3\]"):
        kplanes_tilted_fuse(pts[:, :2], rotations, plane)
    with pytest.raises(ValueError, match=r"rotations \[T, 3, 3\]"):
        kplanes_tilted_fuse(pts, rotations[:, :2, :], plane)
    with pytest.raises(ValueError, match=r"3\*T"):
        kplanes_tilted_fuse(pts, rotations, plane[:3])
    with pytest.raises(TypeError, match="fp32-only"):
        kplanes_tilted_fuse(pts.double(), rotations, plane)


def test_ops_registered_with_reference_names():
    for name in (
        "tv_loss_iso_3d",
        "tv_loss_iso_3d_bwd",
        "tv_loss_sq_3d",
        "tv_loss_sq_3d_bwd",
        "tv_loss_l1_3d",
        "tv_loss_l1_3d_bwd",
        "kplanes_tilted_fuse",
        "kplanes_tilted_fuse_bwd",
        "kplanes_tilted_tv_fuse",
        "kplanes_tilted_tv_fuse_bwd",
    ):
        assert hasattr(torch.ops.quantem_cuda, name)


def test_fake_impls_give_output_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        vol = torch.empty(2, 5, 6, 7)
        assert torch.ops.quantem_cuda.tv_loss_iso_3d(vol, 1e-8).shape == ()
        assert torch.ops.quantem_cuda.tv_loss_l1_3d(vol).shape == (3,)
        loss, grad = torch.ops.quantem_cuda.tv_loss_sq_3d_fwd_grad(vol, torch.empty(1))
        assert loss.shape == () and grad.shape == vol.shape
        out = torch.ops.quantem_cuda.kplanes_tilted_fuse(
            torch.empty(10, 3), torch.empty(2, 3, 3), torch.empty(6, 4, 5, 5)
        )
        assert out.shape == (10, 8)


def test_raw_kplanes_ops_check_what_the_kernels_index():
    """The registered ops (called without the public wrappers) refuse inputs
    that would make a kernel index outside its buffers, before any launch."""
    p, r = torch.rand(5, 3), torch.eye(3).expand(2, 3, 3).contiguous()
    with pytest.raises(ValueError, match=r"plane must be \[3\*T"):
        torch.ops.quantem_cuda.kplanes_tilted_fuse(p, r, torch.rand(5, 4, 6, 6))
    with pytest.raises(ValueError, match=r"rotations must be \[T, 3, 3\]"):
        torch.ops.quantem_cuda.kplanes_tilted_fuse(p, torch.rand(2, 3), torch.rand(6, 4, 6, 6))
    with pytest.raises(ValueError, match=r"pts must be \[B, 3\]"):
        torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(torch.rand(5, 2), r, torch.rand(6, 4, 6, 6), torch.rand(5, 8))
    # host tensors never reach a kernel
    with pytest.raises(ValueError, match="CUDA"):
        torch.ops.quantem_cuda.kplanes_tilted_tv_fuse(p, r, torch.rand(6, 4, 6, 6), 0.1)


def test_product_code_never_reaches_the_oracle():
    """The package and its C sources name no oracle, torch restatement, CPU
    fallback or subprocess: the only compute path is the CUDA extension, and
    an op given CPU tensors raises instead of computing."""
    import re
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    pattern = re.compile(r"^\s*(from|import)\s+(oracle|torch_ref|subprocess|ctypes|numpy)\b", re.M)
    files = [*(root / "quantem-cuda_b200" / "quantem").rglob("*.py")]
    assert files
    for f in files:
        text = f.read_text()
        assert not pattern.search(text), f"{f} imports a CPU path"
    inc = re.compile(r'^\s*#\s*include\s*[<"][^>"]*oracle', re.M)
    for f in (root / "quantem-cuda_b200" / "csrc").glob("*.c*"):
        assert not inc.search(f.read_text()), f"{f} includes oracle code"
