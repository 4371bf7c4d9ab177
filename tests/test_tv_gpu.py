"""GPU parity of the 3-D TV kernels against the CPU oracle, the golden
fixtures, the reference's own CUDA `_core` (when built into oracle/_ref) and
the reference's behavioural tests (tests/core/test_tv_loss.py)."""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from quantem.cuda import _core
    from quantem.cuda.core import (
        ptycho_tv_loss,
        tv_loss_iso_3d,
        tv_loss_iso_3d_fwd_grad,
        tv_loss_l1_3d,
        tv_loss_l1_3d_fwd_grad,
        tv_loss_multi_3d_fwd_grad,
        tv_loss_sq_3d,
        tv_loss_sq_3d_fwd_grad,
    )

# Shapes: the reference's (test_tv_loss.py:10) plus TMA-path shapes with
# partial tiles in H and W, several tiles, odd W (generic path) and a size-1 dim.
SHAPES = [
    (33, 57, 18),
    (3, 32, 32, 32),
    (2, 3, 16, 16, 16),
    (1, 32, 32),
    (2, 40, 70, 260),
    (3, 17, 33, 132),
    (2, 9, 31, 37),
    (1, 64, 64, 64),
    (5, 2, 3, 8),
    (128, 128, 128),  # the single-volume squared-TV benchmark shape
]

FWD_RTOL = 1e-5  # forward tolerance (relative)
GRAD_RTOL = 1e-4  # gradient tolerance (relative, element-wise)


def rand_vol(shape, seed):
    gen = torch.Generator().manual_seed(seed)
    return torch.rand(shape, generator=gen, dtype=torch.float32)


def n_corners(shape):
    b = int(np.prod(shape[:-3])) if len(shape) > 3 else 1
    d, h, w = shape[-3:]
    return max(1, b * (d - 1) * (h - 1) * (w - 1))


def assert_grad_close(actual: torch.Tensor, expected: np.ndarray):
    exp = torch.from_numpy(np.ascontiguousarray(expected)).reshape(actual.shape)
    scale = float(exp.abs().max()) if exp.numel() else 1.0
    torch.testing.assert_close(actual.cpu(), exp, rtol=GRAD_RTOL, atol=1e-6 * max(scale, 1e-30))


@pytest.mark.parametrize("shape", SHAPES)
def test_losses_match_oracle(shape):
    vol = rand_vol(shape, 11)
    v = vol.cuda()
    iso = tv_loss_iso_3d(v, eps=1e-8).item()
    sq = tv_loss_sq_3d(v).item()
    l1 = tv_loss_l1_3d(v).cpu().numpy()
    np.testing.assert_allclose(iso, oracle.tv_iso_loss(vol.numpy(), 1e-8), rtol=FWD_RTOL, atol=1e-12)
    np.testing.assert_allclose(sq, oracle.tv_sq_loss(vol.numpy()), rtol=FWD_RTOL, atol=1e-12)
    np.testing.assert_allclose(l1, oracle.tv_l1_loss(vol.numpy()), rtol=FWD_RTOL, atol=1e-12)


@pytest.mark.parametrize("shape", SHAPES)
def test_autograd_gradients_match_oracle(shape):
    vol = rand_vol(shape, 12)
    x = vol.numpy()
    v = vol.cuda().requires_grad_(True)
    tv_loss_iso_3d(v, eps=1e-6).backward()
    assert_grad_close(v.grad, oracle.tv_iso_grad(x, 1.0 / n_corners(shape), 1e-6))
    v.grad = None
    (2.5 * tv_loss_sq_3d(v)).backward()
    assert_grad_close(v.grad, oracle.tv_sq_grad(x, 2.5))
    v.grad = None
    w = torch.tensor([0.7, 1.3, 0.2], device="cuda")
    (tv_loss_l1_3d(v) * w).sum().backward()
    assert_grad_close(v.grad, oracle.tv_l1_grad(x, [0.7, 1.3, 0.2]))


def assert_same_up_to_rounding(a: torch.Tensor, b: torch.Tensor):
    # The single sweep and the gradient-only kernel evaluate the same formulas;
    # they agree to about 1 ulp of the gradient's scale.
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6 * b.abs().max().item())


@pytest.mark.parametrize("shape", SHAPES)
def test_single_sweep_matches_pair(shape):
    v = rand_vol(shape, 13).cuda()
    loss, grad = tv_loss_iso_3d_fwd_grad(v, 0.5, eps=1e-8)
    vv = v.clone().requires_grad_(True)
    ref = tv_loss_iso_3d(vv, eps=1e-8)
    (0.5 * ref).backward()
    torch.testing.assert_close(loss, ref.detach(), rtol=1e-6, atol=0)
    assert_same_up_to_rounding(grad, vv.grad)

    loss, grad = tv_loss_sq_3d_fwd_grad(v, 3.0)
    vv.grad = None
    (3.0 * tv_loss_sq_3d(vv)).backward()
    torch.testing.assert_close(loss, tv_loss_sq_3d(v), rtol=1e-6, atol=0)
    assert_same_up_to_rounding(grad, vv.grad)

    g3 = (0.7, 1.3, 0.2)
    sums, grad = tv_loss_l1_3d_fwd_grad(v, g3)
    vv.grad = None
    (tv_loss_l1_3d(vv) * torch.tensor(g3, device="cuda")).sum().backward()
    torch.testing.assert_close(sums, tv_loss_l1_3d(v), rtol=1e-6, atol=0)
    assert_same_up_to_rounding(grad, vv.grad)


def test_golden_fixtures(tv_golden):
    names = sorted({k.split("/")[0] for k in tv_golden if not k.startswith("ptycho")})
    for name in names:
        vol = torch.from_numpy(tv_golden[f"{name}/vol"]).cuda()
        iso_ref = float(tv_golden[f"{name}/iso_loss"])
        iso = tv_loss_iso_3d(vol, eps=1e-8).item()
        if np.isnan(iso_ref):
            assert iso == 0.0
        else:
            np.testing.assert_allclose(iso, iso_ref, rtol=FWD_RTOL)
        np.testing.assert_allclose(tv_loss_sq_3d(vol).item(), float(tv_golden[f"{name}/sq_loss"]), rtol=FWD_RTOL)
        np.testing.assert_allclose(tv_loss_l1_3d(vol).cpu().numpy(), tv_golden[f"{name}/l1_sums"], rtol=FWD_RTOL, atol=1e-9)
        v = vol.clone().requires_grad_(True)
        tv_loss_iso_3d(v, eps=1e-6).backward()
        assert_grad_close(v.grad, tv_golden[f"{name}/iso_grad_eps1e-6"])
        v.grad = None
        tv_loss_sq_3d(v).backward()
        assert_grad_close(v.grad, tv_golden[f"{name}/sq_grad"])
        v.grad = None
        (tv_loss_l1_3d(v) * torch.tensor([0.7, 1.3, 0.2], device="cuda")).sum().backward()
        assert_grad_close(v.grad, tv_golden[f"{name}/l1_grad_w0.7_1.3_0.2"])


@pytest.mark.parametrize("key", ["ptycho_16_5.0_0.1", "ptycho_16_5.0_0.0", "ptycho_1_0.0_0.3"])
def test_ptycho_recipe(tv_golden, key):
    wz, wxy = (float(x) for x in key.split("_")[2:4])
    a = torch.from_numpy(tv_golden[f"{key}/array"]).cuda().requires_grad_(True)
    loss = ptycho_tv_loss(a, (wz, wxy))
    torch.testing.assert_close(loss.cpu(), torch.tensor(float(tv_golden[f"{key}/loss"])), rtol=1e-5, atol=1e-7)
    loss.backward()
    torch.testing.assert_close(a.grad.cpu(), torch.from_numpy(tv_golden[f"{key}/grad"]), rtol=1e-4, atol=1e-7)


@pytest.mark.parametrize("weight", [0.5, 0.0])
def test_tv_vol_scaling(weight):
    from quantem.cuda.core import tv_vol_loss

    x = rand_vol((12, 20, 33), 15)
    v = x.cuda().requires_grad_(True)
    loss = tv_vol_loss(v, weight)
    expect = weight * oracle.tv_sq_loss(x.numpy()) / x.numel()
    np.testing.assert_allclose(loss.item(), expect, rtol=FWD_RTOL, atol=1e-12)
    loss.backward()
    ref = oracle.tv_sq_grad(x.numpy(), weight / x.numel())
    assert_grad_close(v.grad, ref)


def test_deterministic_losses():
    v = rand_vol((2, 40, 70, 260), 14).cuda()
    for fn in (lambda x: tv_loss_iso_3d(x), tv_loss_sq_3d, tv_loss_l1_3d):
        a, b = fn(v), fn(v)
        assert torch.equal(a, b)


def test_reference_behaviours():
    # upstream scaling (test_tv_loss.py:77-86)
    vol = rand_vol((16, 16, 16), 4).cuda()
    v1 = vol.clone().requires_grad_(True)
    v2 = vol.clone().requires_grad_(True)
    tv_loss_sq_3d(v1).backward()
    (3.0 * tv_loss_sq_3d(v2)).backward()
    torch.testing.assert_close(v2.grad, 3.0 * v1.grad, rtol=1e-6, atol=1e-8)
    # non-contiguous input (:89-96, :247-251)
    nc = rand_vol((24, 18, 30), 5).cuda().permute(2, 0, 1)
    assert not nc.is_contiguous()
    x = nc.contiguous().cpu().numpy()
    np.testing.assert_allclose(tv_loss_sq_3d(nc).item(), oracle.tv_sq_loss(x), rtol=FWD_RTOL)
    np.testing.assert_allclose(tv_loss_iso_3d(nc).item(), oracle.tv_iso_loss(x, 1e-8), rtol=FWD_RTOL)
    np.testing.assert_allclose(tv_loss_l1_3d(nc).cpu().numpy(), oracle.tv_l1_loss(x), rtol=FWD_RTOL)
    # degenerate dims: iso loss 0 and grad 0 (:99-110), L1 empty axis (:238-244)
    d = rand_vol((1, 32, 32), 6).cuda().requires_grad_(True)
    loss = tv_loss_iso_3d(d)
    assert loss.item() == 0.0
    loss.backward()
    assert torch.all(d.grad == 0)
    assert tv_loss_l1_3d(d.detach())[0].item() == 0.0
    # L1 plateau: sign(0) = 0 (:204-210)
    ones = torch.ones(8, 8, 8, device="cuda", requires_grad=True)
    tv_loss_l1_3d(ones).sum().backward()
    assert torch.all(ones.grad == 0)


def test_torch_compile_fullgraph():
    def loss_fn(v):
        return tv_loss_iso_3d(v, eps=1e-8) + 0.1 * tv_loss_sq_3d(v) + (tv_loss_l1_3d(v) * v.new_tensor([1.0, 0.5, 0.5])).sum()

    compiled = torch.compile(loss_fn, fullgraph=True)
    vol = rand_vol((32, 32, 32), 7).cuda().requires_grad_(True)
    torch.testing.assert_close(compiled(vol), loss_fn(vol), rtol=1e-6, atol=1e-8)


def test_slab_decomposition_reassembles_whole_volume():
    """The D-slab form behind the multi-GPU path: slabs with one-plane halos,
    owned ranges and boundary flags, summed and stitched, equal the whole."""
    B, D, H, W = 2, 23, 37, 136
    vol = rand_vol((B, D, H, W), 15).cuda()
    g = torch.tensor([1.7], device="cuda")
    g3 = torch.tensor([0.3, 1.1, 0.6], device="cuda")
    cuts = [0, 5, 6, 14, 23]
    for variant, gv, n_acc, eps in ((_core.TV_SQ, g, 1, 0.0), (_core.TV_ISO, g, 1, 1e-6), (_core.TV_L1, g3, 3, 0.0)):
        ws = torch.empty(_core.tv_loss_3d_workspace_bytes(0, 0, 0, 0), dtype=torch.uint8, device="cuda")
        whole_acc = torch.zeros(n_acc, device="cuda")
        whole_grad = torch.empty_like(vol)
        st = torch.cuda.current_stream().cuda_stream
        _core.tv_loss_3d_slab_cuda(variant, 3, vol.data_ptr(), gv.data_ptr(), whole_acc.data_ptr(), whole_grad.data_ptr(),
                                   B, D, H, W, 0, D, 0, 0, eps, 1.0, ws.data_ptr(), ws.numel(), st)
        total = torch.zeros(n_acc, dtype=torch.float64, device="cuda")
        stitched = torch.empty_like(vol)
        for lo, hi in zip(cuts[:-1], cuts[1:]):
            has_prev, has_next = lo > 0, hi < D
            slab = torch.zeros((B, hi - lo + 2, H, W), device="cuda")
            slab[:, 1 : hi - lo + 1] = vol[:, lo:hi]
            if has_prev:
                slab[:, 0] = vol[:, lo - 1]
            if has_next:
                slab[:, -1] = vol[:, hi]
            acc = torch.zeros(n_acc, device="cuda")
            grad = torch.full_like(slab, float("nan"))
            _core.tv_loss_3d_slab_cuda(variant, 3, slab.data_ptr(), gv.data_ptr(), acc.data_ptr(), grad.data_ptr(),
                                       B, hi - lo + 2, H, W, 1, hi - lo + 1, int(has_prev), int(has_next), eps, 1.0,
                                       ws.data_ptr(), ws.numel(), st)
            total += acc.double()
            stitched[:, lo:hi] = grad[:, 1 : hi - lo + 1]
            assert torch.isnan(grad[:, 0]).all() and torch.isnan(grad[:, -1]).all()  # halos untouched
        torch.testing.assert_close(total.float(), whole_acc, rtol=1e-6, atol=0)
        torch.testing.assert_close(stitched, whole_grad, rtol=1e-6, atol=1e-12)


def test_c_abi_reference_signatures():
    """Calls the reference-named entry points through the C ABI with the
    reference's argument lists and conventions (pre-zeroed accumulator,
    acc += sum; csrc/ops/core.h:16-78), and the deterministic workspace form."""
    lib = ctypes.CDLL(str(Path(_core.__file__).parent / "libquantem_cuda_b200.so"))
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.tv_loss_sq_3d_cuda.argtypes = [vp, vp, i, i, i, i, vp]
    lib.tv_loss_iso_3d_cuda.argtypes = [vp, vp, i, i, i, i, f, vp]
    lib.tv_loss_l1_3d_cuda.argtypes = [vp, vp, i, i, i, i, vp]
    lib.tv_loss_sq_3d_ws_cuda.argtypes = [vp, vp, i, i, i, i, vp, ctypes.c_size_t, vp]
    lib.tv_loss_iso_3d_grad_cuda.argtypes = [vp, vp, vp, i, i, i, i, f, vp]
    vol = rand_vol((3, 20, 24, 68), 16)
    v = vol.cuda()
    x = vol.numpy()
    st = torch.cuda.current_stream().cuda_stream
    acc = torch.full((1,), 2.0, device="cuda")  # accumulates on top of 2.0
    assert lib.tv_loss_sq_3d_cuda(v.data_ptr(), acc.data_ptr(), 3, 20, 24, 68, st) == 0
    np.testing.assert_allclose(acc.item() - 2.0, oracle.tv_sq_loss(x), rtol=FWD_RTOL)
    acc = torch.zeros(1, device="cuda")
    assert lib.tv_loss_iso_3d_cuda(v.data_ptr(), acc.data_ptr(), 3, 20, 24, 68, f(1e-8), st) == 0
    np.testing.assert_allclose(acc.item(), oracle.tv_iso_sum(x, 1e-8), rtol=FWD_RTOL)
    acc3 = torch.zeros(3, device="cuda")
    assert lib.tv_loss_l1_3d_cuda(v.data_ptr(), acc3.data_ptr(), 3, 20, 24, 68, st) == 0
    np.testing.assert_allclose(acc3.cpu().numpy(), oracle.tv_l1_loss(x), rtol=FWD_RTOL)
    ws = torch.empty(lib.tv_loss_3d_workspace_bytes(0, 0, 0, 0), dtype=torch.uint8, device="cuda")
    acc_ws = [torch.full((1,), 2.0, device="cuda") for _ in range(2)]
    for a in acc_ws:
        assert lib.tv_loss_sq_3d_ws_cuda(v.data_ptr(), a.data_ptr(), 3, 20, 24, 68, ws.data_ptr(), ws.numel(), st) == 0
    np.testing.assert_allclose(acc_ws[0].item() - 2.0, oracle.tv_sq_loss(x), rtol=FWD_RTOL)
    assert torch.equal(acc_ws[0], acc_ws[1])  # fixed-order reduction: the same bits every call
    g = torch.tensor([0.25], device="cuda")
    grad = torch.empty_like(v)
    assert lib.tv_loss_iso_3d_grad_cuda(v.data_ptr(), g.data_ptr(), grad.data_ptr(), 3, 20, 24, 68, f(1e-6), st) == 0
    assert_grad_close(grad, oracle.tv_iso_grad(vol.numpy(), 0.25, 1e-6))


@pytest.mark.skipif(oracle.ref_core() is None, reason="reference _core not built into oracle/_ref")
@pytest.mark.parametrize("shape", [(3, 32, 32, 32), (2, 40, 70, 260), (33, 57, 18)])
def test_matches_reference_cuda_kernels(shape):
    ref = oracle.ref_core()
    v = rand_vol(shape, 17).cuda().reshape(-1, *shape[-3:])
    b, d, h, w = v.shape
    st = torch.cuda.current_stream().cuda_stream
    for name, eps in (("iso", 1e-8), ("sq", None), ("l1", None)):
        acc = torch.zeros(3 if name == "l1" else 1, device="cuda")
        if eps is None:
            getattr(ref, f"tv_loss_{name}_3d_cuda")(v.data_ptr(), acc.data_ptr(), b, d, h, w, st)
        else:
            ref.tv_loss_iso_3d_cuda(v.data_ptr(), acc.data_ptr(), b, d, h, w, eps, st)
        mine = {"iso": lambda: tv_loss_iso_3d(v, eps=1e-8) * n_corners(v.shape), "sq": lambda: tv_loss_sq_3d(v),
                "l1": lambda: tv_loss_l1_3d(v)}[name]()
        torch.testing.assert_close(mine.reshape(-1), acc, rtol=FWD_RTOL, atol=0)
    # gradients
    gs = torch.tensor([0.3], device="cuda")
    g3 = torch.tensor([0.7, 1.3, 0.2], device="cuda")
    for name, gv in (("iso", gs), ("sq", gs), ("l1", g3)):
        ref_grad = torch.zeros_like(v)
        if name == "iso":
            ref.tv_loss_iso_3d_grad_cuda(v.data_ptr(), gv.data_ptr(), ref_grad.data_ptr(), b, d, h, w, 1e-6, st)
            vv = v.clone().requires_grad_(True)
            (tv_loss_iso_3d(vv, eps=1e-6) * (0.3 * n_corners(v.shape))).backward()
        else:
            getattr(ref, f"tv_loss_{name}_3d_grad_cuda")(v.data_ptr(), gv.data_ptr(), ref_grad.data_ptr(), b, d, h, w, st)
            vv = v.clone().requires_grad_(True)
            out = tv_loss_sq_3d(vv) * 0.3 if name == "sq" else (tv_loss_l1_3d(vv) * g3).sum()
            out.backward()
        scale = float(ref_grad.abs().max())
        torch.testing.assert_close(vv.grad, ref_grad, rtol=GRAD_RTOL, atol=1e-6 * scale)


def test_full_size_iso_l1_workload():
    """The benchmark workload: [4, 256, 256, 256] with 1% of voxels equal to
    their +W neighbour (sign(0) = 0 exercised), single-sweep ops vs oracle."""
    gen = torch.Generator().manual_seed(1)
    vol = torch.rand((4, 256, 256, 256), generator=gen)
    flat = vol.view(-1, 256)
    rows = torch.randint(0, flat.shape[0], (vol.numel() // 100,), generator=gen)
    cols = torch.randint(0, 255, rows.shape, generator=gen)
    flat[rows, cols] = flat[rows, cols + 1]
    x = vol.numpy()
    v = vol.cuda()
    loss, grad = tv_loss_iso_3d_fwd_grad(v, 1.0, eps=1e-8)
    np.testing.assert_allclose(loss.item(), oracle.tv_iso_loss(x, 1e-8), rtol=FWD_RTOL)
    assert_grad_close(grad, oracle.tv_iso_grad(x, 1.0 / n_corners(x.shape), 1e-8))
    del grad
    sums, grad = tv_loss_l1_3d_fwd_grad(v, 1.0)
    np.testing.assert_allclose(sums.cpu().numpy(), oracle.tv_l1_loss(x), rtol=FWD_RTOL)
    assert_grad_close(grad, oracle.tv_l1_grad(x, [1.0, 1.0, 1.0]))


def _compare_grad_chunked(grad: torch.Tensor, expected: np.ndarray, planes: int = 32) -> tuple[float, float]:
    """Element-wise gradient check of a large volume, plane slab by plane slab
    (keeps the fp64 temporaries small): |got - expected| <= GRAD_RTOL·|expected|
    + 1e-6·max|expected|. Returns (largest error, largest magnitude)."""
    g = grad.reshape(-1, *grad.shape[-2:])
    e = expected.reshape(-1, *expected.shape[-2:])
    scale = max(float(np.abs(e[k : k + planes]).max()) for k in range(0, e.shape[0], planes))
    worst = 0.0
    for k in range(0, e.shape[0], planes):
        a = g[k : k + planes].cpu().numpy().astype(np.float64)
        b = e[k : k + planes].astype(np.float64)
        err = np.abs(a - b)
        assert np.all(err <= GRAD_RTOL * np.abs(b) + 1e-6 * scale), f"planes {k}..{k + planes}: max err {err.max():.3e}"
        worst = max(worst, float(err.max()))
    return worst, scale


def test_tomography_scale_blob_volume():
    """[1024, 1024, 1024] sum of 64 Gaussian blobs + N(0, 0.01) noise, seed 4
    (the tomography-scale configuration): squared and isotropic loss and
    gradient from the single-sweep ops against the oracle on the whole volume.
    On this smooth field most differences are small against the values, which
    is where the isotropic sweep's approximate square roots would show."""
    import bench

    v = bench.blob_volume(1024, 4, "cuda")
    x = v.cpu().numpy()
    loss, grad = tv_loss_sq_3d_fwd_grad(v, 1.0)
    ref = oracle.tv_sq_loss(x)
    rel = abs(loss.item() - ref) / ref
    assert rel <= FWD_RTOL, rel
    _compare_grad_chunked(grad, oracle.tv_sq_grad(x, 1.0))
    del grad
    loss, grad = tv_loss_iso_3d_fwd_grad(v, 1.0, eps=1e-8)
    ref = oracle.tv_iso_loss(x, 1e-8)
    rel = abs(loss.item() - ref) / ref
    # the loss term uses the MUFU square root (relative error below 2^-22 per
    # term, accumulated in fp64): 1e-5 is the stated tolerance
    assert rel <= FWD_RTOL, rel
    print(f"iso loss rel err on the blob volume: {rel:.3e} (tolerance {FWD_RTOL:g})")
    _compare_grad_chunked(grad, oracle.tv_iso_grad(x, 1.0 / n_corners(x.shape), 1e-8))


MIX_WEIGHTS = {"sq": 0.3, "iso": 1.7, "l1": (0.7, 1.3, 0.2)}
MIX_COMBOS = [("sq", "iso"), ("iso", "l1"), ("sq", "l1"), ("sq", "iso", "l1")]


def _single_terms(v, combo):
    """Losses and the weighted gradient sum from the single-term sweeps."""
    losses, grad = {}, torch.zeros_like(v)
    if "sq" in combo:
        losses["sq"], g = tv_loss_sq_3d_fwd_grad(v, MIX_WEIGHTS["sq"])
        grad += g
    if "iso" in combo:
        losses["iso"], g = tv_loss_iso_3d_fwd_grad(v, MIX_WEIGHTS["iso"], eps=1e-8)
        grad += g
    if "l1" in combo:
        losses["l1"], g = tv_loss_l1_3d_fwd_grad(v, MIX_WEIGHTS["l1"])
        grad += g
    return losses, grad


@pytest.mark.parametrize("combo", MIX_COMBOS, ids=["+".join(c) for c in MIX_COMBOS])
@pytest.mark.parametrize("shape", SHAPES)
def test_multi_term_sweep_matches_single_terms_and_oracle(shape, combo):
    """Two or three terms in one sweep: each loss equals its single-term
    sweep's and the oracle's; the gradient equals the weighted sum of the
    single-term gradients and of the oracle's."""
    vol = rand_vol(shape, 31)
    v = vol.cuda()
    losses, grad = tv_loss_multi_3d_fwd_grad(v, eps=1e-8, **{k: MIX_WEIGHTS[k] for k in combo})
    ref_losses, ref_grad = _single_terms(v, combo)
    assert set(losses) == set(combo)
    for k in combo:
        torch.testing.assert_close(losses[k], ref_losses[k], rtol=1e-6, atol=0)
    assert_same_up_to_rounding(grad, ref_grad)
    x = vol.numpy()
    oracle_grad = np.zeros_like(x.reshape(-1, *x.shape[-3:]))
    if "sq" in combo:
        np.testing.assert_allclose(losses["sq"].item(), oracle.tv_sq_loss(x), rtol=FWD_RTOL)
        oracle_grad += oracle.tv_sq_grad(x, MIX_WEIGHTS["sq"]).reshape(oracle_grad.shape)
    if "iso" in combo:
        np.testing.assert_allclose(losses["iso"].item(), oracle.tv_iso_loss(x, 1e-8), rtol=FWD_RTOL, atol=1e-12)
        oracle_grad += oracle.tv_iso_grad(x, MIX_WEIGHTS["iso"] / n_corners(shape), 1e-8).reshape(oracle_grad.shape)
    if "l1" in combo:
        np.testing.assert_allclose(losses["l1"].cpu().numpy(), oracle.tv_l1_loss(x), rtol=FWD_RTOL)
        oracle_grad += oracle.tv_l1_grad(x, np.array(MIX_WEIGHTS["l1"], np.float32)).reshape(oracle_grad.shape)
    assert_grad_close(grad, oracle_grad)


def test_multi_term_sweep_on_the_benchmark_volume():
    """iso + L1 in one sweep on the [4, 256^3] volume with 1% plateaus (the
    benchmark step done as one sweep instead of two), against the two single
    sweeps and the oracle."""
    import bench

    vol = bench.tv_iso_l1_volume(1)
    v = vol.cuda()
    losses, grad = tv_loss_multi_3d_fwd_grad(v, iso=1.0, l1=1.0, eps=1e-8)
    li, gi = tv_loss_iso_3d_fwd_grad(v, 1.0, eps=1e-8)
    ll, gl = tv_loss_l1_3d_fwd_grad(v, 1.0)
    torch.testing.assert_close(losses["iso"], li, rtol=1e-6, atol=0)
    torch.testing.assert_close(losses["l1"], ll, rtol=1e-6, atol=0)
    assert_same_up_to_rounding(grad, gi + gl)
    x = vol.numpy()
    np.testing.assert_allclose(losses["iso"].item(), oracle.tv_iso_loss(x, 1e-8), rtol=FWD_RTOL)
    np.testing.assert_allclose(losses["l1"].cpu().numpy(), oracle.tv_l1_loss(x), rtol=FWD_RTOL)


def test_multi_term_c_abi_accumulates_and_rejects_one_term():
    lib = ctypes.CDLL(str(Path(_core.__file__).parent / "libquantem_cuda_b200.so"))
    vp, i, f, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    fn = lib.tv_loss_mix_3d_fwd_grad_cuda
    fn.argtypes = [i, i, vp, vp, vp, vp, i, i, i, i, f, f, vp, sz, vp]
    vol = rand_vol((2, 24, 20, 68), 32)
    v = vol.cuda()
    ws = torch.empty(lib.tv_loss_3d_workspace_bytes(0, 0, 0, 0), dtype=torch.uint8, device="cuda")
    g = torch.tensor([0.5, 2.0, 1.0, 1.0, 1.0], device="cuda")
    acc = torch.zeros(5, device="cuda")
    grad = torch.empty_like(v)
    st = torch.cuda.current_stream().cuda_stream
    iso_scale = 0.25  # acc[1] = 0.25 * iso sum; gradient term 2.0 * 0.25 * grad(iso sum)
    for _ in range(2):  # acc += ...
        assert fn(7, 0, v.data_ptr(), g.data_ptr(), acc.data_ptr(), grad.data_ptr(), 2, 24, 20, 68, 1e-8,
                  iso_scale, ws.data_ptr(), ws.numel(), st) == 0
    x = vol.numpy()
    np.testing.assert_allclose(acc[0].item(), 2 * oracle.tv_sq_loss(x), rtol=FWD_RTOL)
    np.testing.assert_allclose(acc[1].item(), 2 * iso_scale * oracle.tv_iso_sum(x, 1e-8), rtol=FWD_RTOL)
    np.testing.assert_allclose(acc[2:].cpu().numpy(), 2 * oracle.tv_l1_loss(x), rtol=FWD_RTOL)
    expected = (oracle.tv_sq_grad(x, 0.5) + oracle.tv_iso_grad(x, 2.0 * iso_scale, 1e-8)
                + oracle.tv_l1_grad(x, np.ones(3, np.float32)))
    assert_grad_close(grad, expected)
    for terms in (0, 1, 2, 4, 8):
        assert fn(terms, 0, v.data_ptr(), g.data_ptr(), acc.data_ptr(), grad.data_ptr(), 2, 24, 20, 68, 1e-8, 1.0,
                  ws.data_ptr(), ws.numel(), st) == 10001


def test_no_kernel_gave_up_waiting():
    torch.cuda.synchronize()
    assert _core.device_fault_word(torch.cuda.current_device()) == 0


def test_first_cuda_work_on_a_fresh_host_thread():
    """The fast path encodes its TMA descriptor through the driver API; it must
    work on a thread that has made no CUDA runtime call yet (autograd runs
    backward on such a thread)."""
    import threading

    v = rand_vol((2, 20, 24, 68), 18).cuda()
    g = torch.ones(1, device="cuda")
    x = v.cpu().numpy()
    # same shapes once on this thread, so that the call on the new thread is
    # served from the caching allocator and issues no torch CUDA call of its own
    tv_loss_iso_3d_fwd_grad(v, g, eps=1e-8)
    torch.cuda.synchronize()
    box = {}

    def work():
        try:
            loss, grad = tv_loss_iso_3d_fwd_grad(v, g, eps=1e-8)
            torch.cuda.synchronize()
            box["res"] = (loss.item(), grad.cpu())
        except Exception as e:  # noqa: BLE001
            box["err"] = e

    th = threading.Thread(target=work)
    th.start()
    th.join()
    assert "err" not in box, box.get("err")
    np.testing.assert_allclose(box["res"][0], oracle.tv_iso_loss(x, 1e-8), rtol=FWD_RTOL)
    assert_grad_close(box["res"][1], oracle.tv_iso_grad(x, 1.0 / n_corners(x.shape), 1e-8))


def test_ops_replay_from_a_cuda_graph():
    """The single-sweep ops and the autograd pair are capturable: a CUDA graph
    replays them with the eager results (workspaces come from torch's
    allocator; per-device setup happens on the first, eager call)."""
    v = rand_vol((2, 24, 40, 132), 16).cuda()
    g = torch.tensor([0.3], device="cuda")
    eager = (tv_loss_iso_3d_fwd_grad(v, g, eps=1e-8), tv_loss_l1_3d(v))
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        (loss, grad), sums = tv_loss_iso_3d_fwd_grad(v, g, eps=1e-8), tv_loss_l1_3d(v)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(loss, eager[0][0]) and torch.equal(grad, eager[0][1]) and torch.equal(sums, eager[1])


class _ReferenceOpLayerCalls:
    """The `_core` calls the reference's TV op layer makes, in its order and
    with its buffers (src/quantem/cuda/core/_ops.py:39-228): a zeroed
    accumulator for each loss (the iso sum then divided by the corner count),
    an upstream scalar (iso: divided by the corner count) and a zero- or
    empty-initialised gradient for each backward. Bound to either `_core`."""

    def __init__(self, core):
        self.core = core

    def _args(self, vol):
        b, d, h, w = vol.shape
        return b, d, h, w, torch.cuda.current_stream().cuda_stream

    def iso(self, vol, eps):
        b, d, h, w, st = self._args(vol)
        acc = torch.zeros(1, dtype=torch.float32, device=vol.device)
        self.core.tv_loss_iso_3d_cuda(vol.data_ptr(), acc.data_ptr(), b, d, h, w, float(eps), st)
        return acc.squeeze(0) / float(n_corners(vol.shape))

    def iso_bwd(self, vol, grad_out, eps):
        b, d, h, w, st = self._args(vol)
        g = (grad_out.reshape(1) / float(n_corners(vol.shape))).contiguous()
        grad = torch.zeros_like(vol)
        self.core.tv_loss_iso_3d_grad_cuda(vol.data_ptr(), g.data_ptr(), grad.data_ptr(), b, d, h, w, float(eps), st)
        return grad

    def sq(self, vol):
        b, d, h, w, st = self._args(vol)
        acc = torch.zeros(1, dtype=torch.float32, device=vol.device)
        self.core.tv_loss_sq_3d_cuda(vol.data_ptr(), acc.data_ptr(), b, d, h, w, st)
        return acc.squeeze(0)

    def sq_bwd(self, vol, grad_out):
        b, d, h, w, st = self._args(vol)
        g = grad_out.reshape(1).contiguous()
        grad = torch.empty_like(vol)
        self.core.tv_loss_sq_3d_grad_cuda(vol.data_ptr(), g.data_ptr(), grad.data_ptr(), b, d, h, w, st)
        return grad

    def l1(self, vol):
        b, d, h, w, st = self._args(vol)
        acc = torch.zeros(3, dtype=torch.float32, device=vol.device)
        self.core.tv_loss_l1_3d_cuda(vol.data_ptr(), acc.data_ptr(), b, d, h, w, st)
        return acc

    def l1_bwd(self, vol, grad_out):
        b, d, h, w, st = self._args(vol)
        g = grad_out.reshape(3).contiguous()
        grad = torch.empty_like(vol)
        self.core.tv_loss_l1_3d_grad_cuda(vol.data_ptr(), g.data_ptr(), grad.data_ptr(), b, d, h, w, st)
        return grad


@pytest.mark.parametrize("shape", [(3, 32, 32, 32), (2, 40, 70, 260), (1, 33, 57, 18), (1, 128, 128, 128)])
def test_reference_op_layer_calls_run_unchanged_on_this_core(shape):
    """The reference's op layer, re-pointed at this `_core`, gives the oracle's
    results; and the same calls on the reference's own `_core` (when built)
    agree with it."""
    x = rand_vol(shape, 23).numpy()
    v = torch.from_numpy(x).cuda()
    eps = 1e-8
    layers = [("here", _ReferenceOpLayerCalls(_core))]
    if oracle.ref_core() is not None:
        layers.append(("reference", _ReferenceOpLayerCalls(oracle.ref_core())))
    up = torch.tensor([0.8], device="cuda")
    up3 = torch.tensor([0.7, 1.3, 0.2], device="cuda")
    results = {}
    for tag, ops in layers:
        results[tag] = (ops.iso(v, eps), ops.sq(v), ops.l1(v), ops.iso_bwd(v, up, 1e-6), ops.sq_bwd(v, up),
                        ops.l1_bwd(v, up3))
    iso, sq, l1, g_iso, g_sq, g_l1 = results["here"]
    np.testing.assert_allclose(iso.item(), oracle.tv_iso_loss(x, eps), rtol=FWD_RTOL)
    np.testing.assert_allclose(sq.item(), oracle.tv_sq_loss(x), rtol=FWD_RTOL)
    np.testing.assert_allclose(l1.cpu().numpy(), oracle.tv_l1_loss(x), rtol=FWD_RTOL)
    assert_grad_close(g_iso, oracle.tv_iso_grad(x, 0.8 / n_corners(shape), 1e-6))
    assert_grad_close(g_sq, oracle.tv_sq_grad(x, 0.8))
    assert_grad_close(g_l1, oracle.tv_l1_grad(x, np.array([0.7, 1.3, 0.2], np.float32)))
    if "reference" in results:
        for mine, theirs in zip(results["here"][:3], results["reference"][:3]):
            torch.testing.assert_close(mine, theirs, rtol=FWD_RTOL, atol=0)
        for mine, theirs in zip(results["here"][3:], results["reference"][3:]):
            scale = theirs.abs().max().item()
            torch.testing.assert_close(mine, theirs, rtol=GRAD_RTOL, atol=1e-6 * scale)
