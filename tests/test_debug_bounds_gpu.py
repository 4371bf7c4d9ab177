"""The bounds-checked build (libquantem_cuda_b200_debug.so, -DQC_DEBUG_BOUNDS)
on the parity shapes: every computed global index is checked against its
buffer, so a clean run here means no kernel indexed outside its buffers on
these inputs (this pool offers no memory sanitizer). The checked build must
also give the release build's results: TV bit for bit, K-Planes forward bit
for bit, K-Planes gradients to atomics-order tolerance.

The checked library runs in a child process of its own: each build links the
CUDA runtime statically, and one process keeps to one of them."""

from __future__ import annotations

import ctypes
from pathlib import Path

import pytest
import multiprocessing as mp

import torch

pytestmark = pytest.mark.gpu

LIBDIR = Path(__file__).resolve().parents[1] / "quantem-cuda_b200" / "quantem" / "cuda"
TV_SHAPES = [(2, 40, 70, 260), (3, 17, 33, 132), (3, 9, 31, 37), (1, 2, 3, 8)]
TV_CASES = ((0, [1.3, 0.0, 0.0]), (1, [0.7, 0.0, 0.0]), (2, [0.7, 1.3, 0.2]))
KP_CFGS = [(2000, 4, 32, 50, 33), (257, 3, 5, 7, 9), (300, 2, 8, 11, 11)]


def _load(name):
    vp, i, f, sz, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_long
    lib = ctypes.CDLL(str(LIBDIR / name))
    lib.tv_loss_3d_slab_cuda.argtypes = [i, i, vp, vp, vp, vp, i, i, i, i, i, i, i, i, f, f, vp, sz, vp]
    lib.kplanes_tilted_fuse_cuda.argtypes = [vp, vp, vp, vp, L, i, i, i, i, vp]
    lib.kplanes_tilted_fuse_grad_cuda.argtypes = [vp] * 7 + [L, i, i, i, i, vp]
    lib.kplanes_tilted_tv_fuse_cuda.argtypes = [vp, vp, vp, vp, L, i, i, i, i, f, vp]
    lib.quantem_cuda_device_fault_word.argtypes = [i, ctypes.POINTER(ctypes.c_uint), i]
    lib.quantem_cuda_last_error.restype = ctypes.c_char_p
    return lib


def _run_all(name):
    """Every case through one library; CPU tensors and the fault word."""
    lib = _load(name)
    st = torch.cuda.current_stream().cuda_stream
    w = ctypes.c_uint(0)
    assert lib.quantem_cuda_device_fault_word(0, ctypes.byref(w), 1) == 0
    res = {}
    for shape in TV_SHAPES:
        vol = torch.rand(shape, generator=torch.Generator().manual_seed(3)).cuda()
        B, D, H, W = shape
        for variant, g in TV_CASES:
            gt = torch.tensor(g, device="cuda")
            acc = torch.zeros(3, device="cuda")
            grad = torch.full_like(vol, float("nan"))
            ws = torch.empty(48 << 10, dtype=torch.uint8, device="cuda")
            status = lib.tv_loss_3d_slab_cuda(variant, 7, vol.data_ptr(), gt.data_ptr(), acc.data_ptr(),
                                              grad.data_ptr(), B, D, H, W, 0, D, 0, 0, 1e-8, 1.0, ws.data_ptr(),
                                              ws.numel(), st)
            assert status == 0, lib.quantem_cuda_last_error()
            torch.cuda.synchronize()
            res[("tv", shape, variant)] = (acc.cpu(), grad.cpu())
    for cfg in KP_CFGS:
        N, T, C, H, W = cfg
        gen = torch.Generator().manual_seed(4)
        # points beyond the border too: taps clamp at the edges
        pts = torch.empty((N, 3)).uniform_(-1.3, 1.3, generator=gen).cuda()
        rot = torch.empty((T, 3, 3)).uniform_(-1, 1, generator=gen).cuda()
        grid = torch.empty((3 * T, H, W, C)).uniform_(0.1, 0.5, generator=gen).cuda()
        up = torch.randn((N, T * C), generator=gen).cuda()
        out = torch.empty((N, T * C), device="cuda")
        assert lib.kplanes_tilted_fuse_cuda(pts.data_ptr(), rot.data_ptr(), grid.data_ptr(), out.data_ptr(),
                                            N, T, C, H, W, st) == 0, lib.quantem_cuda_last_error()
        tv = torch.empty((4, N, T * C), device="cuda")
        assert lib.kplanes_tilted_tv_fuse_cuda(pts.data_ptr(), rot.data_ptr(), grid.data_ptr(), tv.data_ptr(),
                                               N, T, C, H, W, 0.05, st) == 0, lib.quantem_cuda_last_error()
        gg, gr, gp = torch.zeros_like(grid), torch.zeros_like(rot), torch.zeros_like(pts)
        assert lib.kplanes_tilted_fuse_grad_cuda(pts.data_ptr(), rot.data_ptr(), grid.data_ptr(), up.data_ptr(),
                                                 gg.data_ptr(), gr.data_ptr(), gp.data_ptr(), N, T, C, H, W,
                                                 st) == 0, lib.quantem_cuda_last_error()
        torch.cuda.synchronize()
        res[("kp", cfg)] = (out.cpu(), tv.cpu(), gg.cpu(), gr.cpu(), gp.cpu())
    assert lib.quantem_cuda_device_fault_word(0, ctypes.byref(w), 1) == 0
    return res, w.value


def _child(name, queue):
    try:
        res, fault = _run_all(name)
        # numpy arrays travel by value (tensors would be shared through file
        # descriptors that close when this process exits)
        queue.put(("ok", {k: tuple(t.numpy() for t in v) for k, v in res.items()}, fault))
    except BaseException as e:  # report, do not hang the parent
        queue.put(("error", repr(e), 0))


def test_checked_build_is_clean_and_matches_release():
    if not (LIBDIR / "libquantem_cuda_b200_debug.so").exists():
        pytest.fail("libquantem_cuda_b200_debug.so not built (build_ext.build_debug)")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child, args=("libquantem_cuda_b200_debug.so", q))
    p.start()
    kind, checked, fault = q.get(timeout=600)
    p.join(timeout=60)
    assert kind == "ok", checked
    assert fault == 0, f"bounds checks fired: fault word {fault:#x}"
    release, rel_fault = _run_all("libquantem_cuda_b200.so")
    assert rel_fault == 0
    for key, ref in release.items():
        got = tuple(torch.from_numpy(a) for a in checked[key])
        if key[0] == "tv":
            assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1]), key
        else:
            assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1]), key
            for a, b in zip(ref[2:], got[2:]):
                torch.testing.assert_close(b, a, rtol=1e-4, atol=1e-5 * a.abs().max().item())
