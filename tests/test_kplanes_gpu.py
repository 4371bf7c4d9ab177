"""GPU parity of the fused tilted K-Planes kernels against the CPU oracle,
the golden fixtures (the reference's grid_sample definition), the reference's
own CUDA `_core` (when built into oracle/_ref) and the reference's behavioural
tests (tests/core/ml/test_kplanes_tilted.py)."""

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
    from quantem.cuda.core.ml import kplanes_tilted_fuse

# (N, T, C, H, W): the reference's configs (test_kplanes_tilted.py:18-23) and
# every vector width of the fast path (C = 4, 8, 16, 32, 64, 128), plus C not
# a multiple of 4 and C above 128 (scalar path).
CONFIGS = [
    (37, 1, 1, 5, 5),
    (257, 3, 5, 7, 9),
    (4096, 4, 8, 200, 200),
    (2000, 8, 32, 50, 33),
    (777, 4, 4, 11, 13),
    (1000, 2, 16, 20, 30),
    (600, 2, 64, 17, 9),
    (300, 3, 128, 16, 16),
    (200, 2, 132, 8, 8),
]

FWD_RTOL = 1e-5


def make_inputs(N, T, C, H, W, seed, pts_scale=1.1):
    gen = torch.Generator().manual_seed(seed)
    pts = torch.empty((N, 3)).uniform_(-pts_scale, pts_scale, generator=gen)
    rot = torch.empty((T, 3, 3)).uniform_(-1.0, 1.0, generator=gen)
    plane = torch.empty((3 * T, C, H, W)).uniform_(0.1, 0.5, generator=gen)
    up = torch.randn((N, T * C), generator=gen)
    return pts, rot, plane, up


def grads(pts, rot, plane, up):
    inp = [t.cuda().requires_grad_(True) for t in (pts, rot, plane)]
    out = kplanes_tilted_fuse(*inp)
    (out * up.cuda()).sum().backward()
    return out.detach(), [t.grad for t in inp]


def assert_rel_max(actual: torch.Tensor, expected: np.ndarray, rel: float, what: str):
    """Gradient check against the gradient's largest magnitude: atomic
    reductions add a plane cell's contributions in a different order than the
    oracle, so an element that is a near-cancelling sum can carry an error
    that is large against itself but not against the gradient's scale."""
    exp = torch.from_numpy(np.ascontiguousarray(expected)).double()
    err = (actual.detach().cpu().double() - exp).abs().max().item()
    scale = exp.abs().max().item()
    assert err <= rel * max(scale, 1e-30), f"{what}: max err {err:.3e} vs scale {scale:.3e}"


# Element-wise gradient check: every entry whose magnitude is at least
# FLOOR_FRAC of the gradient's largest is within GRAD_RTOL of itself.
GRAD_RTOL = 1e-4
FLOOR_FRAC = 1e-2


def assert_rel_elementwise(actual: torch.Tensor, expected: np.ndarray, what: str, rel: float = GRAD_RTOL,
                           floor_frac: float = FLOOR_FRAC) -> float:
    a = actual.detach().cpu().double().numpy().reshape(-1)
    e = np.ascontiguousarray(expected, dtype=np.float64).reshape(-1)
    floor = floor_frac * np.abs(e).max()
    big = np.abs(e) >= floor
    err = np.abs(a[big] - e[big]) / np.abs(e[big])
    worst = float(err.max()) if err.size else 0.0
    assert worst <= rel, f"{what}: {int((err > rel).sum())} of {int(big.sum())} entries above the floor exceed rel {rel}"
    return worst


@pytest.mark.parametrize("cfg", CONFIGS)
def test_forward_matches_oracle(cfg):
    pts, rot, plane, _ = make_inputs(*cfg, seed=1)
    out = kplanes_tilted_fuse(pts.cuda(), rot.cuda(), plane.cuda()).cpu()
    ref = torch.from_numpy(oracle.kplanes_fwd(pts.numpy(), rot.numpy(), plane.numpy()))
    # the oracle evaluates the same fp32 operations in the same fused order:
    # the forward is bit-exact
    torch.testing.assert_close(out, ref, rtol=0, atol=0)


@pytest.mark.parametrize("cfg", CONFIGS)
def test_gradients_match_oracle(cfg):
    pts, rot, plane, up = make_inputs(*cfg, seed=2)
    _, (gp, gr, gg) = grads(pts, rot, plane, up)
    o_gp, o_gr, o_gg = oracle.kplanes_bwd(pts.numpy(), rot.numpy(), plane.numpy(), up.numpy())
    # gradient tolerance rel 1e-4 (atomics reorder sums), measured against each
    # gradient's largest magnitude
    assert_rel_max(gg, o_gg, 1e-4, "grad_plane")
    assert_rel_max(gp, o_gp, 1e-4, "grad_pts")
    assert_rel_max(gr, o_gr, 1e-4, "grad_rotations")
    for mine, theirs, what in ((gg, o_gg, "grad_plane"), (gp, o_gp, "grad_pts"), (gr, o_gr, "grad_rotations")):
        assert_rel_elementwise(mine, theirs, what)


def ray_points(n_rays: int, samples: int, seed: int, scale: float = 1.1) -> torch.Tensor:
    """Points in runs along rays, laid out as a tomography ray sampler lays
    them out: neighbouring entries share plane cells."""
    gen = torch.Generator().manual_seed(seed)
    xy = torch.empty((n_rays, 1, 2)).uniform_(-scale, scale, generator=gen)
    z = torch.linspace(-scale, scale, samples).view(1, -1, 1)
    return torch.cat([xy.expand(-1, samples, -1), z.expand(n_rays, -1, -1)], dim=-1).reshape(-1, 3).contiguous()


@pytest.mark.parametrize("C", [4, 8, 32])
def test_ray_points_gradients_match_oracle(C):
    """Runs of points that share plane cells, which the backward adds up in
    registers before reducing (at C <= 8): one level, four taps and two levels
    in one launch, against the oracle."""
    from quantem.cuda.core.ml import kplanes_tilted_fuse_levels

    T, H, W = 3, 40, 40
    pts = ray_points(48, 64, seed=81)
    N = pts.shape[0]
    gen = torch.Generator().manual_seed(82)
    rot = torch.empty((T, 3, 3)).uniform_(-1.0, 1.0, generator=gen)
    plane = torch.empty((3 * T, C, H, W)).uniform_(0.1, 0.5, generator=gen)
    up = torch.randn((N, T * C), generator=gen)
    _, (gp, gr, gg) = grads(pts, rot, plane, up)
    o_gp, o_gr, o_gg = oracle.kplanes_bwd(pts.numpy(), rot.numpy(), plane.numpy(), up.numpy())
    for mine, theirs, what in ((gg, o_gg, "grad_plane"), (gp, o_gp, "grad_pts"), (gr, o_gr, "grad_rotations")):
        assert_rel_max(mine, theirs, 1e-4, what)
        assert_rel_elementwise(mine, theirs, what)

    up4 = torch.randn((4, N, T * C), generator=gen)
    _, (gp, gr, gg) = tv_grads(pts, rot, plane, up4, 0.02)
    o_gp, o_gr, o_gg = oracle.kplanes_tv_bwd(pts.numpy(), rot.numpy(), plane.numpy(), up4.numpy(), 0.02)
    for mine, theirs, what in ((gg, o_gg, "four-tap grad_plane"), (gp, o_gp, "four-tap grad_pts"),
                               (gr, o_gr, "four-tap grad_rotations")):
        assert_rel_max(mine, theirs, 1e-4, what)

    planes = [plane, torch.empty((3 * T, C, 24, 24)).uniform_(0.1, 0.5, generator=gen)]
    ups = [up, torch.randn((N, T * C), generator=gen)]
    p = pts.cuda().requires_grad_(True)
    pls = [pl.cuda().requires_grad_(True) for pl in planes]
    outs = kplanes_tilted_fuse_levels(p, rot.cuda(), pls)
    sum(((o * u.cuda()).sum() for o, u in zip(outs, ups))).backward()
    o_gp = np.zeros(pts.shape, dtype=np.float64)
    for lv, (pl, u) in enumerate(zip(planes, ups)):
        g_p, _, g_g = oracle.kplanes_bwd(pts.numpy(), rot.numpy(), pl.numpy(), u.numpy())
        assert_rel_max(pls[lv].grad, g_g, 1e-4, f"grad_plane level {lv}")
        assert_rel_elementwise(pls[lv].grad, g_g, f"grad_plane level {lv}")
        o_gp += g_p
    assert_rel_max(p.grad, o_gp, 1e-4, "grad_pts (sum over levels)")


def test_golden_fixtures_fp64_anchored(kp_golden):
    """test_kplanes_tilted.py:71-95 on the committed fixtures: the kernel's
    error against fp64 torch is no worse than 2x torch's own fp32 error."""
    names = sorted({k.split("/")[0] for k in kp_golden if not k.startswith("border")})
    for name in names:
        t = {k: torch.from_numpy(kp_golden[f"{name}/{k}"]) for k in ("pts", "rotations", "plane", "upstream")}
        out, got = grads(t["pts"], t["rotations"], t["plane"], t["upstream"])
        torch.testing.assert_close(out.cpu(), torch.from_numpy(kp_golden[f"{name}/out_f32"]), rtol=1e-4, atol=5e-6)
        for label, mine in zip(("pts", "rotations", "plane"), got):
            ref64 = kp_golden[f"{name}/grad_{label}_f64"]
            err_torch = np.abs(kp_golden[f"{name}/grad_{label}_f32"].astype(np.float64) - ref64).max()
            err_kernel = np.abs(mine.cpu().double().numpy() - ref64).max()
            assert err_kernel <= max(2.0 * err_torch, 1e-6), (name, label, err_kernel, err_torch)


def test_points_exactly_on_border(kp_golden):
    pts, rot, plane = (torch.from_numpy(kp_golden[f"border/{k}"]).cuda() for k in ("pts", "rotations", "plane"))
    p = pts.clone().requires_grad_(True)
    out = kplanes_tilted_fuse(p, rot, plane)
    torch.testing.assert_close(out.cpu(), torch.from_numpy(kp_golden["border/out_f32"]), rtol=1e-5, atol=1e-6)
    (g,) = torch.autograd.grad(out.sum(), p)
    torch.testing.assert_close(g.cpu(), torch.from_numpy(kp_golden["border/grad_pts_f32"]), rtol=1e-4, atol=1e-6)
    # with rotations requiring grad too (test_kplanes_tilted.py:118-128)
    r = rot.clone().requires_grad_(True)
    p2 = pts.clone().requires_grad_(True)
    out2 = kplanes_tilted_fuse(p2, r, plane)
    (g2,) = torch.autograd.grad(out2.sum(), p2)
    torch.testing.assert_close(g2.cpu(), torch.from_numpy(kp_golden["border/grad_pts_f32"]), rtol=1e-4, atol=1e-6)


def test_upstream_grad_scaling():
    pts, rot, plane, _ = make_inputs(64, 2, 4, 9, 9, seed=3)
    pl = plane.cuda().requires_grad_(True)
    p, r = pts.cuda(), rot.cuda()
    kplanes_tilted_fuse(p, r, pl).sum().backward()
    g1 = pl.grad.clone()
    pl.grad = None
    (kplanes_tilted_fuse(p, r, pl) * 3.0).sum().backward()
    torch.testing.assert_close(pl.grad, g1 * 3.0, rtol=1e-5, atol=1e-6)


def test_non_contiguous_and_channels_last_inputs():
    pts, rot, plane, up = make_inputs(128, 2, 8, 9, 11, seed=4)
    p, r, pl = pts.cuda(), rot.cuda(), plane.cuda()
    ref = kplanes_tilted_fuse(p, r, pl)
    pts_nc = p.t().contiguous().t()
    plane_nc = pl.permute(0, 1, 3, 2).contiguous().permute(0, 1, 3, 2)
    assert not pts_nc.is_contiguous() and not plane_nc.is_contiguous()
    torch.testing.assert_close(kplanes_tilted_fuse(pts_nc, r, plane_nc), ref, rtol=0, atol=0)
    # a channels-last parameter takes the no-copy path, and its gradient keeps
    # the parameter's layout
    plane_cl = pl.contiguous(memory_format=torch.channels_last).requires_grad_(True)
    out = kplanes_tilted_fuse(p, r, plane_cl)
    torch.testing.assert_close(out, ref, rtol=0, atol=0)
    (out * up.cuda()).sum().backward()
    plane_c = pl.clone().requires_grad_(True)
    (kplanes_tilted_fuse(p, r, plane_c) * up.cuda()).sum().backward()
    assert plane_cl.grad.stride() == plane_cl.stride()
    torch.testing.assert_close(plane_cl.grad, plane_c.grad, rtol=1e-5, atol=1e-7)


def test_compile_fullgraph():
    pts, rot, plane, _ = make_inputs(512, 2, 4, 17, 17, seed=5)
    p, r, g = (t.cuda().requires_grad_(True) for t in (pts, rot, plane))

    @torch.compile(fullgraph=True)
    def f(a, b, c):
        return kplanes_tilted_fuse(a, b, c).square().mean()

    f(p, r, g).backward()
    assert p.grad is not None and r.grad is not None and g.grad is not None


def test_eager_path_matches_registered_ops():
    """The public wrappers' eager path (autograd.Function) and the registered
    torch.library ops give the same outputs bit for bit and the same
    gradients (to the reordering of atomic sums), for the single-level,
    four-tap and multi-level ops."""
    from quantem.cuda.core.ml import kplanes_tilted_fuse_levels, kplanes_tilted_tv_fuse

    pts, rot, plane, up = make_inputs(3000, 3, 8, 30, 26, seed=17)
    plane2 = torch.empty((9, 8, 12, 15)).uniform_(0.1, 0.5, generator=torch.Generator().manual_seed(18))
    up4 = torch.randn((4, *up.shape), generator=torch.Generator().manual_seed(19))
    ops = torch.ops.quantem_cuda
    cases = [
        ("one level", lambda a, b, c, d: [kplanes_tilted_fuse(a, b, c)],
         lambda a, b, c, d: [ops.kplanes_tilted_fuse(a, b, c)], [up]),
        ("four taps", lambda a, b, c, d: [kplanes_tilted_tv_fuse(a, b, c, 0.03)],
         lambda a, b, c, d: [ops.kplanes_tilted_tv_fuse(a, b, c, 0.03)], [up4]),
        ("two levels", lambda a, b, c, d: kplanes_tilted_fuse_levels(a, b, [c, d]),
         lambda a, b, c, d: ops.kplanes_tilted_fuse_levels(a, b, [c, d]), [up, up]),
    ]
    for what, eager, registered, ups in cases:
        results = []
        for fn in (eager, registered):
            leaves = [t.cuda().requires_grad_(True) for t in (pts, rot, plane, plane2)]
            outs = fn(*leaves)
            sum((o * u.cuda()).sum() for o, u in zip(outs, ups)).backward()
            results.append(([o.detach() for o in outs], [x.grad for x in leaves]))
        (outs_e, grads_e), (outs_r, grads_r) = results
        for a, b in zip(outs_e, outs_r):
            assert torch.equal(a, b), what
        for name, a, b in zip(("pts", "rotations", "plane", "plane2"), grads_e, grads_r):
            assert (a is None) == (b is None), (what, name)
            if a is not None:
                torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5 * b.abs().max().item(), msg=f"{what} {name}")


def test_input_validation_on_device():
    pts, rot, plane, _ = make_inputs(16, 2, 4, 9, 9, seed=6)
    pts, rot, plane = pts.cuda(), rot.cuda(), plane.cuda()
    with pytest.raises(ValueError, match=r"pts \[B, 3\]"):
        kplanes_tilted_fuse(pts[:, :2], rot, plane)
    with pytest.raises(ValueError, match=r"rotations \[T, 3, 3\]"):
        kplanes_tilted_fuse(pts, rot[:, :2, :], plane)
    with pytest.raises(ValueError, match=r"3\*T"):
        kplanes_tilted_fuse(pts, rot, plane[:3])
    with pytest.raises(TypeError, match="fp32-only"):
        kplanes_tilted_fuse(pts.double(), rot, plane)


def test_empty_point_set():
    pts, rot, plane, _ = make_inputs(0, 2, 8, 9, 9, seed=7)
    p = pts.cuda().requires_grad_(True)
    pl = plane.cuda().requires_grad_(True)
    out = kplanes_tilted_fuse(p, rot.cuda(), pl)
    assert out.shape == (0, 16)
    out.sum().backward()
    assert torch.all(pl.grad == 0)


def test_c_abi_accumulates_like_the_reference():
    """kplanes_tilted_fuse_grad_cuda accumulates into ggrid, gR and gpts:
    two calls on the same buffers give twice the gradient."""
    lib = ctypes.CDLL(str(Path(_core.__file__).parent / "libquantem_cuda_b200.so"))
    vp, i, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_long
    lib.kplanes_tilted_fuse_grad_cuda.argtypes = [vp] * 7 + [L, i, i, i, i, vp]
    N, T, C, H, W = 500, 3, 32, 19, 23
    pts, rot, plane, up = make_inputs(N, T, C, H, W, seed=8)
    p, r, go = pts.cuda(), rot.cuda(), up.cuda()
    grid_cl = plane.cuda().permute(0, 2, 3, 1).contiguous()
    gg = torch.zeros_like(grid_cl)
    gr = torch.zeros_like(r)
    gp = torch.zeros_like(p)
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        assert lib.kplanes_tilted_fuse_grad_cuda(p.data_ptr(), r.data_ptr(), grid_cl.data_ptr(), go.data_ptr(),
                                                 gg.data_ptr(), gr.data_ptr(), gp.data_ptr(), N, T, C, H, W, st) == 0
    o_gp, o_gr, o_gg = oracle.kplanes_bwd(pts.numpy(), rot.numpy(), plane.numpy(), up.numpy())
    assert_rel_max(gg.permute(0, 3, 1, 2), 2 * o_gg, 1e-4, "2x grad_plane")
    assert_rel_max(gr, 2 * o_gr, 1e-4, "2x grad_rotations")
    assert_rel_max(gp, 2 * o_gp, 1e-4, "2x grad_pts")


@pytest.mark.skipif(oracle.ref_core() is None, reason="reference _core not built into oracle/_ref")
@pytest.mark.parametrize("cfg", [(4096, 4, 8, 200, 200), (2000, 8, 32, 50, 33), (257, 3, 5, 7, 9)])
def test_matches_reference_cuda_kernels(cfg):
    ref = oracle.ref_core()
    N, T, C, H, W = cfg
    pts, rot, plane, up = make_inputs(*cfg, seed=9)
    p, r, go = pts.cuda(), rot.cuda(), up.cuda()
    grid_cl = plane.cuda().permute(0, 2, 3, 1).contiguous()
    st = torch.cuda.current_stream().cuda_stream
    ref_out = torch.empty((N, T * C), device="cuda")
    ref.kplanes_tilted_fuse_cuda(p.data_ptr(), r.data_ptr(), grid_cl.data_ptr(), ref_out.data_ptr(), N, T, C, H, W, st)
    out = kplanes_tilted_fuse(p, r, plane.cuda())
    torch.testing.assert_close(out, ref_out, rtol=0, atol=0)  # bit-exact with the reference kernel
    gg = torch.zeros_like(grid_cl)
    gr = torch.zeros_like(r)
    gp = torch.zeros_like(p)
    ref.kplanes_tilted_fuse_grad_cuda(p.data_ptr(), r.data_ptr(), grid_cl.data_ptr(), go.data_ptr(), gg.data_ptr(),
                                      gr.data_ptr(), gp.data_ptr(), N, T, C, H, W, st)
    _, (m_gp, m_gr, m_gg) = grads(pts, rot, plane, up)
    for mine, theirs, what in ((m_gg, gg.permute(0, 3, 1, 2), "plane"), (m_gr, gr, "rotations"), (m_gp, gp, "pts")):
        err = (mine - theirs).abs().max().item()
        assert err <= 1e-4 * theirs.abs().max().item(), (what, err)


def _bench_inputs(seed, N, T, C, res):
    import bench

    return bench.kplanes_inputs(seed, N=N, T=T, C=C, res=res)


def test_benchmark_scale_full_parity():
    """The single-level benchmark configuration at full size: N = 2^20 points
    U[-1, 1]^3, 4 rotations from normalised quaternions, C = 32, 256x256
    planes U[0.1, 0.5], upstream N(0, 1), seed 2. Forward bit-exact with the
    oracle on every point; plane, rotation and point gradients against the
    oracle's fp64 backward over all points, both against the gradient's
    largest magnitude and element by element above the magnitude floor."""
    pts, rot, plane, up = _bench_inputs(2, 1 << 20, 4, 32, 256)
    p, r, pl, go = pts.cuda(), rot.cuda(), plane.cuda(), up.cuda()
    out = kplanes_tilted_fuse(p, r, pl)
    ref = oracle.kplanes_fwd(pts.numpy(), rot.numpy(), plane.numpy())
    assert np.array_equal(out.cpu().numpy(), ref), "forward differs from the oracle"
    del out, ref
    g_pts, g_rot, g_plane = torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, pl, go)
    o_gp, o_gr, o_gg = oracle.kplanes_bwd(pts.numpy(), rot.numpy(), plane.numpy(), up.numpy())
    for mine, theirs, what in ((g_plane, o_gg, "grad_plane"), (g_rot, o_gr, "grad_rotations"), (g_pts, o_gp, "grad_pts")):
        assert_rel_max(mine, theirs, GRAD_RTOL, what)
        assert_rel_elementwise(mine, theirs, what)
    # linearity in the upstream gradient
    g2 = torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, pl, 2 * go)
    for a, b in zip((g_pts, g_rot, g_plane), g2):
        assert_rel_max(b, (2 * a).cpu().numpy(), 1e-5, "linearity")


def test_multiscale_finest_level_parity():
    """The multiscale configuration's finest level (512x512 planes, 8
    rotations from normalised quaternions, C = 32, seed 3) on the first 2^18
    of its 2^24 points: forward bit-exact, gradients within rel 1e-4."""
    n_total, T, C = 1 << 24, 8, 32
    import bench

    gen = torch.Generator().manual_seed(3)
    pts = torch.empty((n_total, 3)).uniform_(-1.0, 1.0, generator=gen)[: 1 << 18].clone()
    rot = bench.quaternion_rotations(T, gen)
    for res in (64, 128, 256):  # the coarser levels' planes come first in the stream
        torch.empty((3 * T, C, res, res)).uniform_(0.1, 0.5, generator=gen)
    plane = torch.empty((3 * T, C, 512, 512)).uniform_(0.1, 0.5, generator=gen)
    up = torch.randn((pts.shape[0], T * C), generator=torch.Generator().manual_seed(33))
    p, r, pl, go = pts.cuda(), rot.cuda(), plane.cuda(), up.cuda()
    out = kplanes_tilted_fuse(p, r, pl)
    ref = oracle.kplanes_fwd(pts.numpy(), rot.numpy(), plane.numpy())
    assert np.array_equal(out.cpu().numpy(), ref), "forward differs from the oracle"
    del out, ref
    g_pts, g_rot, g_plane = torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, pl, go)
    o_gp, o_gr, o_gg = oracle.kplanes_bwd(pts.numpy(), rot.numpy(), plane.numpy(), up.numpy())
    for mine, theirs, what in ((g_plane, o_gg, "grad_plane"), (g_rot, o_gr, "grad_rotations"), (g_pts, o_gp, "grad_pts")):
        assert_rel_max(mine, theirs, GRAD_RTOL, what)
        assert_rel_elementwise(mine, theirs, what)


@pytest.mark.parametrize("shape", [(12, 32, 256, 256), (6, 8, 17, 20), (3, 5, 7, 9), (6, 132, 8, 8), (2, 40, 33, 36)])
def test_plane_layout_transposes(shape):
    """[P, C, H, W] <-> [P, H, W, C], tiled fast path (C, H*W multiples of 4) and
    the general path, against torch's permute."""
    P, C, H, W = shape
    gen = torch.Generator().manual_seed(10)
    x = torch.rand(shape, generator=gen).cuda()
    cl = torch.empty((P, H, W, C), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _core.kplanes_planes_to_channels_last_cuda(x.data_ptr(), cl.data_ptr(), P, C, H, W, st)
    assert torch.equal(cl, x.permute(0, 2, 3, 1))
    back = torch.empty_like(x)
    _core.kplanes_planes_from_channels_last_cuda(cl.data_ptr(), back.data_ptr(), P, C, H, W, st)
    assert torch.equal(back, x)


@pytest.mark.parametrize("cfg", [(2000, 4, 32, 50, 33), (500, 3, 5, 9, 7), (300, 2, 16, 16, 16)])
@pytest.mark.parametrize("channels_last", [False, True])
@pytest.mark.parametrize("buckets", [1, 2, 4])
def test_per_rotation_backward_matches_whole_backward(cfg, channels_last, buckets):
    """The multi-GPU path's per-rotation backward (one launch per rotation of
    kplanes_tilted_fuse_grad_rotations_cuda, each rotation's plane gradient put
    back in the parameter's layout at once) against the op on all rotations."""
    from quantem.cuda import sharded

    N, T, C, H, W = cfg
    pts, rot, plane, up = make_inputs(N, T, C, H, W, seed=41)
    p, r, u = pts.cuda(), rot.cuda(), up.cuda()
    g = plane.cuda()
    if channels_last:
        g = g.contiguous(memory_format=torch.channels_last)
    out, g_pts, g_rot, g_plane, works = sharded._kplanes_fwd_bwd_bucketed(p, r, g, u, None, 1, buckets)
    assert works == []
    ref_out = torch.ops.quantem_cuda.kplanes_tilted_fuse(p, r, g)
    ref_pts, ref_rot, ref_plane = torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, g, u)
    assert torch.equal(out, ref_out)
    # plane and rotation gradients are accumulated in the same order per
    # rotation; the point gradient sums the rotations in another order
    torch.testing.assert_close(g_plane, ref_plane, rtol=1e-5, atol=1e-6 * ref_plane.abs().max().item())
    torch.testing.assert_close(g_rot, ref_rot, rtol=1e-4, atol=1e-5 * ref_rot.abs().max().item())
    torch.testing.assert_close(g_pts, ref_pts, rtol=1e-4, atol=1e-5 * ref_pts.abs().max().item())
    assert g_plane.stride() == ref_plane.stride()


def test_rotation_range_validation():
    z = torch.zeros(16, device="cuda")
    with pytest.raises(RuntimeError, match="rotations \\[2, 5\\) outside \\[0, 4\\)"):
        _core.kplanes_tilted_fuse_grad_rotations_cuda(*(z.data_ptr(),) * 7, 1, 4, 4, 2, 2, 2, 5,
                                                     torch.cuda.current_stream().cuda_stream)


# ── four-tap variant (kplanes_tilted_tv_fuse) ────────────────────────────────

# the reference's tv configs (test_kplanes_tilted.py:191-197) and the fast path
# at C = 4, 16, 64, 128
TV_CONFIGS = [
    (37, 1, 1, 5, 5),
    (257, 3, 5, 7, 9),
    (1024, 4, 8, 50, 50),
    (2000, 4, 32, 33, 33),
    (500, 2, 4, 20, 30),
    (300, 3, 16, 16, 12),
    (200, 2, 64, 9, 17),
    (100, 2, 128, 8, 8),
]


def tv_grads(pts, rot, plane, up, h):
    from quantem.cuda.core.ml import kplanes_tilted_tv_fuse

    inp = [t.cuda().requires_grad_(True) for t in (pts, rot, plane)]
    out = kplanes_tilted_tv_fuse(*inp, h=h)
    (out * up.cuda()).sum().backward()
    return out.detach(), [t.grad for t in inp]


@pytest.mark.parametrize("cfg", TV_CONFIGS)
def test_tv_forward_matches_oracle_and_base(cfg):
    from quantem.cuda.core.ml import kplanes_tilted_tv_fuse

    pts, rot, plane, _ = make_inputs(*cfg, seed=42)
    p, r, g = pts.cuda(), rot.cuda(), plane.cuda()
    out = kplanes_tilted_tv_fuse(p, r, g, h=0.05)
    assert out.shape == (4, cfg[0], cfg[1] * cfg[2])
    # tap 0 is the base op, bit for bit (test_kplanes_tilted.py:224-233)
    torch.testing.assert_close(out[0], kplanes_tilted_fuse(p, r, g), rtol=0, atol=0)
    ref = torch.from_numpy(oracle.kplanes_tv_fwd(pts.numpy(), rot.numpy(), plane.numpy(), 0.05))
    torch.testing.assert_close(out.cpu(), ref, rtol=0, atol=0)


@pytest.mark.parametrize("cfg", TV_CONFIGS)
def test_tv_gradients_match_oracle(cfg):
    N, T, C, H, W = cfg
    pts, rot, plane, _ = make_inputs(*cfg, seed=43)
    up = torch.randn((4, N, T * C), generator=torch.Generator().manual_seed(5))
    _, (gp, gr, gg) = tv_grads(pts, rot, plane, up, 0.02)
    o_gp, o_gr, o_gg = oracle.kplanes_tv_bwd(pts.numpy(), rot.numpy(), plane.numpy(), up.numpy(), 0.02)
    assert_rel_max(gg, o_gg, 1e-4, "grad_plane")
    assert_rel_max(gp, o_gp, 1e-4, "grad_pts")
    assert_rel_max(gr, o_gr, 1e-4, "grad_rotations")


def test_tv_golden_fixtures_fp64_anchored(kp_tv_golden):
    """test_kplanes_tilted.py:249-286 on the committed fixtures (K = 4 for
    rotations, 2 elsewhere)."""
    names = sorted({k.split("/")[0] for k in kp_tv_golden if not k.startswith("tv_border")})
    for name in names:
        t = {k: torch.from_numpy(kp_tv_golden[f"{name}/{k}"]) for k in ("pts", "rotations", "plane", "upstream")}
        h = float(kp_tv_golden[f"{name}/h"])
        out, got = tv_grads(t["pts"], t["rotations"], t["plane"], t["upstream"], h)
        torch.testing.assert_close(out.cpu(), torch.from_numpy(kp_tv_golden[f"{name}/out_f32"]), rtol=1e-4, atol=5e-6)
        for label, mine in zip(("pts", "rotations", "plane"), got):
            ref64 = kp_tv_golden[f"{name}/grad_{label}_f64"]
            err_torch = np.abs(kp_tv_golden[f"{name}/grad_{label}_f32"].astype(np.float64) - ref64).max()
            err_kernel = np.abs(mine.cpu().double().numpy() - ref64).max()
            k = 4.0 if label == "rotations" else 2.0
            assert err_kernel <= max(k * err_torch, 1e-6), (name, label, err_kernel, err_torch)


def test_tv_border_points(kp_tv_golden):
    from quantem.cuda.core.ml import kplanes_tilted_tv_fuse

    pts, rot, plane = (torch.from_numpy(kp_tv_golden[f"tv_border/{k}"]).cuda() for k in ("pts", "rotations", "plane"))
    h = float(kp_tv_golden["tv_border/h"])
    p = pts.clone().requires_grad_(True)
    out = kplanes_tilted_tv_fuse(p, rot, plane, h=h)
    torch.testing.assert_close(out.cpu(), torch.from_numpy(kp_tv_golden["tv_border/out_f32"]), rtol=1e-4, atol=1e-6)
    (g,) = torch.autograd.grad(out.sum(), p)
    assert torch.isfinite(g).all()
    torch.testing.assert_close(g.cpu(), torch.from_numpy(kp_tv_golden["tv_border/grad_pts_f32"]), rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("h_val", [2.0, 1e-4])
def test_tv_edge_case_h(h_val):
    from quantem.cuda.core.ml import kplanes_tilted_tv_fuse

    pts, rot, plane, _ = make_inputs(256, 2, 8, 17, 17, seed=55)
    inp = [t.cuda().requires_grad_(True) for t in (pts, rot, plane)]
    out = kplanes_tilted_tv_fuse(*inp, h=h_val)
    assert torch.isfinite(out).all()
    out.sum().backward()
    for t in inp:
        assert torch.isfinite(t.grad).all()


def test_tv_compile_fullgraph():
    from quantem.cuda.core.ml import kplanes_tilted_tv_fuse

    pts, rot, plane, _ = make_inputs(512, 2, 4, 17, 17, seed=56)
    inp = [t.cuda().requires_grad_(True) for t in (pts, rot, plane)]

    @torch.compile(fullgraph=True)
    def f(p, r, g):
        return kplanes_tilted_tv_fuse(p, r, g, h=0.01).square().mean()

    f(*inp).backward()
    assert all(t.grad is not None for t in inp)


def test_tv_input_validation():
    from quantem.cuda.core.ml import kplanes_tilted_tv_fuse

    pts, rot, plane, _ = make_inputs(16, 2, 4, 9, 9, seed=57)
    p, r, g = pts.cuda(), rot.cuda(), plane.cuda()
    with pytest.raises(ValueError, match=r"pts \[B, 3\]"):
        kplanes_tilted_tv_fuse(p[:, :2], r, g, h=0.01)
    with pytest.raises(ValueError, match=r"rotations \[T, 3, 3\]"):
        kplanes_tilted_tv_fuse(p, r[:, :2, :], g, h=0.01)
    with pytest.raises(ValueError, match=r"3\*T"):
        kplanes_tilted_tv_fuse(p, r, g[:3], h=0.01)
    with pytest.raises(TypeError, match="fp32-only"):
        kplanes_tilted_tv_fuse(p.double(), r, g, h=0.01)


def test_tv_channels_last_plane_and_empty_points():
    from quantem.cuda.core.ml import kplanes_tilted_tv_fuse

    pts, rot, plane, up4 = make_inputs(300, 2, 8, 9, 11, seed=58)
    up = torch.randn((4, 300, 16), generator=torch.Generator().manual_seed(6))
    _, (gp, gr, gg) = tv_grads(pts, rot, plane, up, 0.03)
    cl = plane.cuda().contiguous(memory_format=torch.channels_last).requires_grad_(True)
    p, r = pts.cuda().requires_grad_(True), rot.cuda().requires_grad_(True)
    (kplanes_tilted_tv_fuse(p, r, cl, h=0.03) * up.cuda()).sum().backward()
    torch.testing.assert_close(cl.grad, gg, rtol=1e-5, atol=1e-6 * gg.abs().max().item())
    assert cl.grad.stride() == cl.stride()
    empty = kplanes_tilted_tv_fuse(pts[:0].cuda(), rot.cuda(), plane.cuda(), h=0.03)
    assert empty.shape == (4, 0, 16)


@pytest.mark.skipif(oracle.ref_core() is None, reason="reference _core not built into oracle/_ref")
@pytest.mark.parametrize("cfg", [(2000, 4, 32, 33, 33), (257, 3, 5, 7, 9)])
def test_tv_matches_reference_cuda_kernels(cfg):
    from quantem.cuda.core.ml import kplanes_tilted_tv_fuse

    ref = oracle.ref_core()
    N, T, C, H, W = cfg
    h = 0.05
    pts, rot, plane, _ = make_inputs(*cfg, seed=59)
    up = torch.randn((4, N, T * C), generator=torch.Generator().manual_seed(7)).cuda()
    p, r = pts.cuda(), rot.cuda()
    grid_cl = plane.cuda().permute(0, 2, 3, 1).contiguous()
    st = torch.cuda.current_stream().cuda_stream
    ref_out = torch.empty((4, N, T * C), device="cuda")
    ref.kplanes_tilted_tv_fuse_cuda(p.data_ptr(), r.data_ptr(), grid_cl.data_ptr(), ref_out.data_ptr(), N, T, C, H, W,
                                    h, st)
    out = kplanes_tilted_tv_fuse(p, r, plane.cuda(), h=h)
    torch.testing.assert_close(out, ref_out, rtol=0, atol=0)  # bit-exact with the reference kernel
    gg = torch.zeros_like(grid_cl)
    gr = torch.zeros_like(r)
    gp = torch.zeros_like(p)
    ref.kplanes_tilted_tv_fuse_grad_cuda(p.data_ptr(), r.data_ptr(), grid_cl.data_ptr(), up.data_ptr(), gg.data_ptr(),
                                         gr.data_ptr(), gp.data_ptr(), N, T, C, H, W, h, st)
    _, (m_gp, m_gr, m_gg) = tv_grads(pts, rot, plane, up.cpu(), h)
    for mine, theirs, what in ((m_gg, gg.permute(0, 3, 1, 2), "plane"), (m_gr, gr, "rotations"), (m_gp, gp, "pts")):
        err = (mine - theirs).abs().max().item()
        assert err <= 1e-4 * theirs.abs().max().item(), (what, err)


def test_ops_replay_from_a_cuda_graph():
    pts, rot, plane, up = make_inputs(1000, 2, 32, 24, 20, seed=61)
    p, r, g, u = pts.cuda(), rot.cuda(), plane.cuda(), up.cuda()
    eager_out = torch.ops.quantem_cuda.kplanes_tilted_fuse(p, r, g)
    eager_grads = torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, g, u)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = torch.ops.quantem_cuda.kplanes_tilted_fuse(p, r, g)
        grads = torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, g, u)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager_out)
    for a, b in zip(grads, eager_grads):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5 * b.abs().max().item())


def test_raw_ops_refuse_mismatched_buffers_before_launch():
    """An upstream gradient of the wrong size, or a plane left on the host,
    would make the kernels read outside their buffers: the ops raise first."""
    p = torch.rand(64, 3, device="cuda") * 2 - 1
    r = torch.eye(3, device="cuda").expand(2, 3, 3).contiguous()
    g = torch.rand(6, 8, 5, 5, device="cuda")
    with pytest.raises(ValueError, match="grad_out must have shape"):
        torch.ops.quantem_cuda.kplanes_tilted_fuse_bwd(p, r, g, torch.rand(64, 15, device="cuda"))
    with pytest.raises(ValueError, match="grad_out must have shape"):
        torch.ops.quantem_cuda.kplanes_tilted_tv_fuse_bwd(p, r, g, torch.rand(64, 16, device="cuda"), 0.1)
    with pytest.raises(ValueError, match="all inputs must be on"):
        torch.ops.quantem_cuda.kplanes_tilted_fuse(p, r, g.cpu())
    torch.cuda.synchronize()


# ── several levels in one launch (kplanes_tilted_fuse_levels) ────────────────

# (N, T, C, resolutions): fast path at C = 32 and 8 with levels of different
# (also non-square) sizes, and C = 5 (general per-level fallback)
LEVEL_CONFIGS = [
    (3000, 4, 32, [(16, 16), (32, 32), (64, 48)]),
    (1500, 2, 8, [(9, 13), (33, 17)]),
    (700, 3, 5, [(7, 9), (12, 12)]),
]


def _level_inputs(N, T, C, res, seed):
    gen = torch.Generator().manual_seed(seed)
    pts = torch.empty((N, 3)).uniform_(-1.1, 1.1, generator=gen)
    rot = torch.empty((T, 3, 3)).uniform_(-1.0, 1.0, generator=gen)
    planes = [torch.empty((3 * T, C, h, w)).uniform_(0.1, 0.5, generator=gen) for h, w in res]
    ups = [torch.randn((N, T * C), generator=gen) for _ in res]
    return pts, rot, planes, ups


@pytest.mark.parametrize("cfg", LEVEL_CONFIGS, ids=["c32x3", "c8x2", "c5x2"])
def test_levels_in_one_launch_match_single_level_ops_and_oracle(cfg):
    from quantem.cuda.core.ml import kplanes_tilted_fuse_levels

    N, T, C, res = cfg
    pts, rot, planes, ups = _level_inputs(N, T, C, res, seed=71)
    p = pts.cuda().requires_grad_(True)
    r = rot.cuda().requires_grad_(True)
    pls = [pl.cuda().requires_grad_(True) for pl in planes]
    outs = kplanes_tilted_fuse_levels(p, r, pls)
    sum(((o * u.cuda()).sum() for o, u in zip(outs, ups))).backward()
    o_gp = np.zeros_like(pts.numpy(), dtype=np.float64)
    o_gr = np.zeros_like(rot.numpy(), dtype=np.float64)
    for lv, (out, pl, up) in enumerate(zip(outs, planes, ups)):
        single = kplanes_tilted_fuse(pts.cuda(), rot.cuda(), pl.cuda())
        assert torch.equal(out.detach(), single), f"level {lv} differs from the single-level op"
        ref = oracle.kplanes_fwd(pts.numpy(), rot.numpy(), pl.numpy())
        assert np.array_equal(out.detach().cpu().numpy(), ref), f"level {lv} differs from the oracle"
        gp, gr, gg = oracle.kplanes_bwd(pts.numpy(), rot.numpy(), pl.numpy(), up.numpy())
        assert_rel_max(pls[lv].grad, gg, 1e-4, f"grad_plane level {lv}")
        assert_rel_elementwise(pls[lv].grad, gg, f"grad_plane level {lv}")
        o_gp += gp
        o_gr += gr
    assert_rel_max(p.grad, o_gp, 1e-4, "grad_pts (sum over levels)")
    assert_rel_elementwise(p.grad, o_gp, "grad_pts (sum over levels)")
    assert_rel_max(r.grad, o_gr, 1e-4, "grad_rotations (sum over levels)")


def test_levels_validation():
    from quantem.cuda.core.ml import kplanes_tilted_fuse_levels

    pts, rot, planes, ups = _level_inputs(64, 2, 8, [(9, 9), (5, 7)], seed=72)
    p, r = pts.cuda(), rot.cuda()
    g = [pl.cuda() for pl in planes]
    with pytest.raises(ValueError, match="same channel count"):
        kplanes_tilted_fuse_levels(p, r, [g[0], g[1][:, :4].contiguous()])
    with pytest.raises(ValueError, match="1 to 8 levels"):
        torch.ops.quantem_cuda.kplanes_tilted_fuse_levels(p, r, g * 5)
    with pytest.raises(ValueError, match="3\\*T"):
        kplanes_tilted_fuse_levels(p, r, [g[0], g[1][:3]])
    with pytest.raises(ValueError, match="grad_out must have shape"):
        torch.ops.quantem_cuda.kplanes_tilted_fuse_levels_bwd(p, r, g, [u.cuda()[:, :3] for u in ups])
