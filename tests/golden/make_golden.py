"""Generates the golden fixtures in this directory from the reference's own
pure-torch definitions of the hot path.

The reference (quantem-cuda) pins its kernels against torch functions that
live in its test files:
    tests/core/test_tv_loss.py:13-27      tv_iso_ref, tv_sq_ref
    tests/core/test_tv_loss.py:144-167    tv_l1_ref, ptycho_tv_ref
    tests/core/ml/test_kplanes_tilted.py:26-40  reference (einsum + grid_sample)
    tests/core/ml/test_kplanes_tilted.py:200-220 reference_tv (four taps)
This script imports those modules from a checkout of the reference (its root
given as the first argument or in $QUANTEM_CUDA_REFERENCE), runs them on CPU
with seeded CPU-generated inputs, and stores inputs, outputs and autograd
gradients as .npz files. The fixtures are committed; the tests read only the
.npz files.

    QUANTEM_CUDA_REFERENCE=<quantem-cuda checkout> python tests/golden/make_golden.py
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF: Path | None = None


def _reference_root() -> Path:
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QUANTEM_CUDA_REFERENCE")
    if not root or not (Path(root) / "tests" / "core").is_dir():
        raise SystemExit(
            "make_golden.py: give the quantem-cuda checkout as the first argument or in "
            "$QUANTEM_CUDA_REFERENCE (a directory holding tests/core/)"
        )
    return Path(root)


def _import_reference_tests():
    # The reference test modules import the (GPU-only) package at import time;
    # the functions used here are pure torch, so stub the package names.
    for name in ("quantem", "quantem.cuda", "quantem.cuda.core", "quantem.cuda.core.ml"):
        sys.modules.setdefault(name, types.ModuleType(name))
    core = sys.modules["quantem.cuda.core"]
    ml = sys.modules["quantem.cuda.core.ml"]
    for attr in ("tv_loss_iso_3d", "tv_loss_l1_3d", "tv_loss_sq_3d"):
        setattr(core, attr, None)
    for attr in ("kplanes_tilted_fuse", "kplanes_tilted_tv_fuse"):
        setattr(ml, attr, None)

    def load(rel):
        spec = importlib.util.spec_from_file_location(Path(rel).stem + "_reference", REF / rel)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod

    return load("tests/core/test_tv_loss.py"), load("tests/core/ml/test_kplanes_tilted.py")


# TV shapes: the reference test shapes (test_tv_loss.py:10) scaled to keep the
# fixtures small, a 5-D input, the degenerate size-1 case (:99-110) and a
# volume with exact zero W-differences (sign(0) = 0 in the L1 gradient).
TV_CASES = [
    ("ref_33x57x18", (33, 57, 18), 0, False),
    ("batched_3x16x16x16", (3, 16, 16, 16), 1, False),
    ("five_d_2x3x8x12x16", (2, 3, 8, 12, 16), 2, False),
    ("degenerate_1x32x32", (1, 32, 32), 3, False),
    ("plateaus_2x12x16x20", (2, 12, 16, 20), 4, True),
    ("odd_w_4x9x7x13", (4, 9, 7, 13), 5, False),
]

# K-Planes (N, T, C, H, W): reference test configs (test_kplanes_tilted.py:18-23)
# with the large ones scaled down, plus C=32 and C=8 cases on the fast path.
KP_CASES = [
    ("ref_37_1_1_5_5", (37, 1, 1, 5, 5), 0),
    ("ref_257_3_5_7_9", (257, 3, 5, 7, 9), 1),
    ("c8_300_4_8_16_16", (300, 4, 8, 16, 16), 2),
    ("c32_500_2_32_20_13", (500, 2, 32, 20, 13), 3),
]


def make_tv(tvmod) -> dict:
    out = {}
    for name, shape, seed, plateaus in TV_CASES:
        gen = torch.Generator().manual_seed(1000 + seed)
        vol = torch.rand(shape, generator=gen, dtype=torch.float32)
        if plateaus:
            # 1% of voxels (w < W-1) copy their +W neighbour: dw == 0 exactly.
            flat = vol.reshape(-1, shape[-1])
            rows = torch.randint(0, flat.shape[0], (max(1, flat.numel() // 100),), generator=gen)
            cols = torch.randint(0, shape[-1] - 1, rows.shape, generator=gen)
            flat[rows, cols] = flat[rows, cols + 1]
        out[f"{name}/vol"] = vol.numpy()
        # forward values
        out[f"{name}/iso_loss"] = np.float64(tvmod.tv_iso_ref(vol.double(), eps=1e-8).item())
        out[f"{name}/sq_loss"] = np.float64(tvmod.tv_sq_ref(vol.double()).item())
        out[f"{name}/l1_sums"] = tvmod.tv_l1_ref(vol.double()).numpy()
        out[f"{name}/iso_loss_f32"] = np.float32(tvmod.tv_iso_ref(vol, eps=1e-8).item())
        out[f"{name}/sq_loss_f32"] = np.float32(tvmod.tv_sq_ref(vol).item())
        # gradients (fp32 torch autograd, as the reference's tests compare against)
        v = vol.clone().requires_grad_(True)
        tvmod.tv_iso_ref(v, eps=1e-6).backward()
        out[f"{name}/iso_grad_eps1e-6"] = v.grad.numpy()
        v = vol.clone().requires_grad_(True)
        tvmod.tv_sq_ref(v).backward()
        out[f"{name}/sq_grad"] = v.grad.numpy()
        v = vol.clone().requires_grad_(True)
        weights = torch.tensor([0.7, 1.3, 0.2])
        (tvmod.tv_l1_ref(v) * weights).sum().backward()
        out[f"{name}/l1_grad_w0.7_1.3_0.2"] = v.grad.numpy()
    # ptychography recipe (test_tv_loss.py:213-235): loss and gradient
    for num_slices, weight in [(16, (5.0, 0.1)), (16, (5.0, 0.0)), (1, (0.0, 0.3))]:
        gen = torch.Generator().manual_seed(77 + num_slices)
        arr = torch.rand((num_slices, 24, 20), generator=gen)
        a = arr.clone().requires_grad_(True)
        loss = tvmod.ptycho_tv_ref(a, weight)
        loss.backward()
        key = f"ptycho_{num_slices}_{weight[0]}_{weight[1]}"
        out[f"{key}/array"] = arr.numpy()
        out[f"{key}/loss"] = np.float32(loss.item())
        out[f"{key}/grad"] = a.grad.numpy()
    return out


def make_kplanes(kpmod) -> dict:
    out = {}
    for name, (N, T, C, H, W), seed in KP_CASES:
        gen = torch.Generator().manual_seed(2000 + seed)
        pts = torch.empty((N, 3)).uniform_(-1.1, 1.1, generator=gen)
        rot = torch.empty((T, 3, 3)).uniform_(-1.0, 1.0, generator=gen)
        plane = torch.empty((3 * T, C, H, W)).uniform_(0.1, 0.5, generator=gen)
        upstream = torch.randn((N, T * C), generator=gen)
        for k, t in (("pts", pts), ("rotations", rot), ("plane", plane), ("upstream", upstream)):
            out[f"{name}/{k}"] = t.numpy()
        for dtype, tag in ((torch.float32, "f32"), (torch.float64, "f64")):
            inp = tuple(t.to(dtype).requires_grad_(True) for t in (pts, rot, plane))
            res = kpmod.reference(*inp)
            gp, gr, gg = torch.autograd.grad((res * upstream.to(dtype)).sum(), inp)
            out[f"{name}/out_{tag}"] = res.detach().numpy()
            out[f"{name}/grad_pts_{tag}"] = gp.numpy()
            out[f"{name}/grad_rotations_{tag}"] = gr.numpy()
            out[f"{name}/grad_plane_{tag}"] = gg.numpy()
    # points exactly on and beyond the border (test_kplanes_tilted.py:98-128)
    T, C, H, W = 2, 3, 11, 11
    gen = torch.Generator().manual_seed(7)
    rot = torch.stack([torch.eye(3), torch.eye(3).roll(1, 0)]).float()
    plane = torch.empty((3 * T, C, H, W)).uniform_(0.1, 0.5, generator=gen)
    pts = torch.tensor(
        [[-1.0, -1.0, -1.0], [1.0, 1.0, 1.0], [-1.0, 1.0, 0.0], [0.0, -1.0, 1.0], [2.0, 0.5, -3.0]]
    )
    p = pts.clone().requires_grad_(True)
    res = kpmod.reference(p, rot, plane)
    (gp,) = torch.autograd.grad(res.sum(), p)
    out["border/pts"] = pts.numpy()
    out["border/rotations"] = rot.numpy()
    out["border/plane"] = plane.numpy()
    out["border/out_f32"] = res.detach().numpy()
    out["border/grad_pts_f32"] = gp.numpy()
    return out


# four-tap K-Planes (N, T, C, H, W, h): the reference's tv test configs
# (test_kplanes_tilted.py:191-197) scaled down, the fast path at C=8 and C=32,
# and a border case whose taps cross the edge (:289-322).
KP_TV_CASES = [
    ("tv_37_1_1_5_5", (37, 1, 1, 5, 5), 0.05, 0),
    ("tv_257_3_5_7_9", (257, 3, 5, 7, 9), 0.02, 1),
    ("tv_c8_200_4_8_12_12", (200, 4, 8, 12, 12), 0.05, 2),
    ("tv_c32_300_2_32_17_13", (300, 2, 32, 17, 13), 0.02, 3),
]


def make_kplanes_tv(kpmod) -> dict:
    out = {}
    for name, (N, T, C, H, W), h, seed in KP_TV_CASES:
        gen = torch.Generator().manual_seed(3000 + seed)
        pts = torch.empty((N, 3)).uniform_(-1.1, 1.1, generator=gen)
        rot = torch.empty((T, 3, 3)).uniform_(-1.0, 1.0, generator=gen)
        plane = torch.empty((3 * T, C, H, W)).uniform_(0.1, 0.5, generator=gen)
        upstream = torch.randn((4, N, T * C), generator=gen)
        out[f"{name}/h"] = np.float32(h)
        for k, t in (("pts", pts), ("rotations", rot), ("plane", plane), ("upstream", upstream)):
            out[f"{name}/{k}"] = t.numpy()
        for dtype, tag in ((torch.float32, "f32"), (torch.float64, "f64")):
            inp = tuple(t.to(dtype).requires_grad_(True) for t in (pts, rot, plane))
            res = kpmod.reference_tv(*inp, h=h)
            gp, gr, gg = torch.autograd.grad((res * upstream.to(dtype)).sum(), inp)
            out[f"{name}/out_{tag}"] = res.detach().numpy()
            out[f"{name}/grad_pts_{tag}"] = gp.numpy()
            out[f"{name}/grad_rotations_{tag}"] = gr.numpy()
            out[f"{name}/grad_plane_{tag}"] = gg.numpy()
    T, C, H, W, h = 2, 4, 11, 11, 0.05
    gen = torch.Generator().manual_seed(13)
    rot = torch.stack([torch.eye(3), torch.eye(3).roll(1, 0)]).float()
    plane = torch.empty((3 * T, C, H, W)).uniform_(0.1, 0.5, generator=gen)
    pts = torch.tensor([[-1.0, -1.0, -1.0], [1.0, 1.0, 1.0], [0.98, 0.0, 0.0], [0.0, 0.98, 0.0],
                        [0.0, 0.0, 0.98], [2.0, -3.0, 0.5]])
    p = pts.clone().requires_grad_(True)
    res = kpmod.reference_tv(p, rot, plane, h=h)
    (gp,) = torch.autograd.grad(res.sum(), p)
    out["tv_border/h"] = np.float32(h)
    out["tv_border/pts"] = pts.numpy()
    out["tv_border/rotations"] = rot.numpy()
    out["tv_border/plane"] = plane.numpy()
    out["tv_border/out_f32"] = res.detach().numpy()
    out["tv_border/grad_pts_f32"] = gp.numpy()
    return out


def main() -> None:
    global REF
    REF = _reference_root()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    tvmod, kpmod = _import_reference_tests()
    np.savez_compressed(HERE / "tv_golden.npz", **make_tv(tvmod))
    np.savez_compressed(HERE / "kplanes_golden.npz", **make_kplanes(kpmod))
    np.savez_compressed(HERE / "kplanes_tv_golden.npz", **make_kplanes_tv(kpmod))
    for f in ("tv_golden.npz", "kplanes_golden.npz", "kplanes_tv_golden.npz"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
