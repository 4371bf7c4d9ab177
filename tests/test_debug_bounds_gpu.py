"""The bounds-checked build (libquantem_cuda_b200_debug.so, -DQC_DEBUG_BOUNDS)
on the parity shapes: every computed global index is checked against its
buffer, so a clean run here means no kernel indexed outside its buffers on
these inputs (this pool offers no memory sanitizer). The checked build must
also give the release build's results: TV bit for bit, K-Planes forward bit
for bit, K-Planes gradients to atomics-order tolerance."""

from __future__ import annotations

import ctypes
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

LIBDIR = Path(__file__).resolve().parents[1] / "quantem-cuda_b200" / "quantem" / "cuda"
vp, i, f, sz, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_long


def _load(name):
    lib = ctypes.CDLL(str(LIBDIR / name))
    lib.tv_loss_3d_slab_cuda.argtypes = [i, i, vp, vp, vp, vp, i, i, i, i, i, i, i, i, f, f, vp, sz, vp]
    lib.kplanes_tilted_fuse_cuda.argtypes = [vp, vp, vp, vp, L, i, i, i, i, vp]
    lib.kplanes_tilted_fuse_grad_cuda.argtypes = [vp] * 7 + [L, i, i, i, i, vp]
    lib.kplanes_tilted_tv_fuse_cuda.argtypes = [vp, vp, vp, vp, L, i, i, i, i, f, vp]
    lib.quantem_cuda_device_fault_word.argtypes = [i, ctypes.POINTER(ctypes.c_uint), i]
    lib.quantem_cuda_last_error.restype = ctypes.c_char_p
    return lib


@pytest.fixture(scope="module")
def libs():
    if not (LIBDIR / "libquantem_cuda_b200_debug.so").exists():
        pytest.fail("libquantem_cuda_b200_debug.so not built (build_ext.build_debug)")
    return _load("libquantem_cuda_b200.so"), _load("libquantem_cuda_b200_debug.so")


def _fault(lib) -> int:
    w = ctypes.c_uint(0)
    assert lib.quantem_cuda_device_fault_word(0, ctypes.byref(w), 1) == 0
    return w.value


def _tv(lib, variant, vol, g, Dp_range=None):
    B, D, H, W = vol.shape
    acc = torch.zeros(3, device="cuda")
    grad = torch.full_like(vol, float("nan"))
    ws = torch.empty(48 << 10, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.tv_loss_3d_slab_cuda(variant, 7, vol.data_ptr(), g.data_ptr(), acc.data_ptr(), grad.data_ptr(),
                                    B, D, H, W, 0, D, 0, 0, 1e-8, 1.0, ws.data_ptr(), ws.numel(), st) == 0, \
        lib.quantem_cuda_last_error()
    torch.cuda.synchronize()
    return acc, grad


@pytest.mark.parametrize("shape", [(2, 40, 70, 260), (3, 17, 33, 132), (3, 9, 31, 37), (1, 2, 3, 8)])
def test_tv_checked_build_is_clean_and_identical(libs, shape):
    rel, dbg = libs
    _fault(dbg)
    vol = torch.rand(shape, generator=torch.Generator().manual_seed(3)).cuda()
    for variant, g in ((0, [1.3]), (1, [0.7]), (2, [0.7, 1.3, 0.2])):
        gt = torch.tensor(g + [0.0] * (3 - len(g)), device="cuda")
        a_r, g_r = _tv(rel, variant, vol, gt)
        a_d, g_d = _tv(dbg, variant, vol, gt)
        assert torch.equal(a_r, a_d) and torch.equal(g_r, g_d), variant
    assert _fault(dbg) == 0


@pytest.mark.parametrize("cfg", [(2000, 4, 32, 50, 33), (257, 3, 5, 7, 9), (300, 2, 8, 11, 11)])
def test_kplanes_checked_build_is_clean_and_identical(libs, cfg):
    rel, dbg = libs
    _fault(dbg)
    N, T, C, H, W = cfg
    gen = torch.Generator().manual_seed(4)
    # points beyond the border too: taps clamp at the edges
    pts = torch.empty((N, 3)).uniform_(-1.3, 1.3, generator=gen).cuda()
    rot = torch.empty((T, 3, 3)).uniform_(-1, 1, generator=gen).cuda()
    grid = torch.empty((3 * T, H, W, C)).uniform_(0.1, 0.5, generator=gen).cuda()
    up = torch.randn((N, T * C), generator=gen).cuda()
    st = torch.cuda.current_stream().cuda_stream
    outs, grads = [], []
    for lib in (rel, dbg):
        out = torch.empty((N, T * C), device="cuda")
        assert lib.kplanes_tilted_fuse_cuda(pts.data_ptr(), rot.data_ptr(), grid.data_ptr(), out.data_ptr(),
                                            N, T, C, H, W, st) == 0
        tv = torch.empty((4, N, T * C), device="cuda")
        assert lib.kplanes_tilted_tv_fuse_cuda(pts.data_ptr(), rot.data_ptr(), grid.data_ptr(), tv.data_ptr(),
                                               N, T, C, H, W, 0.05, st) == 0
        gg, gr, gp = torch.zeros_like(grid), torch.zeros_like(rot), torch.zeros_like(pts)
        assert lib.kplanes_tilted_fuse_grad_cuda(pts.data_ptr(), rot.data_ptr(), grid.data_ptr(), up.data_ptr(),
                                                 gg.data_ptr(), gr.data_ptr(), gp.data_ptr(), N, T, C, H, W, st) == 0
        torch.cuda.synchronize()
        outs.append((out, tv))
        grads.append((gg, gr, gp))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    for a, b in zip(*grads):
        torch.testing.assert_close(b, a, rtol=1e-4, atol=1e-5 * a.abs().max().item())
    assert _fault(dbg) == 0
