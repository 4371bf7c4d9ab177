"""Pins the CPU oracle (oracle/) against golden vectors produced by the
reference's own pure-torch definitions (tests/golden/make_golden.py)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle

from conftest import golden_cases


def _tv_names(tv_golden):
    return [c for c in golden_cases(tv_golden) if not c.startswith("ptycho")]


def test_tv_losses_match_reference_definitions(tv_golden):
    for name in _tv_names(tv_golden):
        vol = tv_golden[f"{name}/vol"]
        iso_ref = tv_golden[f"{name}/iso_loss"]
        if np.isnan(iso_ref):
            # torch's mean over an empty corner set is NaN; the op's contract
            # is loss 0 (reference test_tv_loss.py:99-107).
            assert oracle.tv_iso_loss(vol, 1e-8) == 0.0
        else:
            np.testing.assert_allclose(oracle.tv_iso_loss(vol, 1e-8), iso_ref, rtol=1e-6, atol=1e-9)
        np.testing.assert_allclose(oracle.tv_sq_loss(vol), tv_golden[f"{name}/sq_loss"], rtol=1e-6, atol=1e-9)
        np.testing.assert_allclose(oracle.tv_l1_loss(vol), tv_golden[f"{name}/l1_sums"], rtol=1e-6, atol=1e-9)


def test_tv_gradients_match_reference_definitions(tv_golden):
    for name in _tv_names(tv_golden):
        vol = tv_golden[f"{name}/vol"]
        v4 = vol.reshape(-1, *vol.shape[-3:])
        b, d, h, w = v4.shape
        n = max(1, b * (d - 1) * (h - 1) * (w - 1))
        np.testing.assert_allclose(
            oracle.tv_iso_grad(vol, 1.0 / n, 1e-6), tv_golden[f"{name}/iso_grad_eps1e-6"], rtol=1e-4, atol=1e-7
        )
        np.testing.assert_allclose(oracle.tv_sq_grad(vol, 1.0), tv_golden[f"{name}/sq_grad"], rtol=1e-4, atol=1e-6)
        np.testing.assert_allclose(
            oracle.tv_l1_grad(vol, [0.7, 1.3, 0.2]), tv_golden[f"{name}/l1_grad_w0.7_1.3_0.2"], rtol=1e-4, atol=1e-6
        )


def test_degenerate_and_plateau_known_answers(tv_golden):
    vol = tv_golden["degenerate_1x32x32/vol"]
    assert oracle.tv_iso_sum(vol, 1e-8) == 0.0
    assert np.all(oracle.tv_iso_grad(vol, 1.0, 1e-8) == 0.0)
    assert oracle.tv_l1_loss(vol)[0] == 0.0
    ones = np.ones((8, 8, 8), np.float32)
    assert np.all(oracle.tv_l1_grad(ones, [1.0, 1.0, 1.0]) == 0.0)  # sign(0) = 0


@pytest.mark.parametrize("key", ["ptycho_16_5.0_0.1", "ptycho_16_5.0_0.0", "ptycho_1_0.0_0.3"])
def test_ptycho_recipe_from_l1_sums(tv_golden, key):
    arr = tv_golden[f"{key}/array"]
    wz, wxy = (float(x) for x in key.split("_")[2:4])
    s, h, w = arr.shape
    sums = oracle.tv_l1_loss(arr)
    counts = np.maximum(np.array([(s - 1) * h * w, s * (h - 1) * w, s * h * (w - 1)], np.float64), 1)
    wt = np.array([wz, wxy, wxy])
    active = max(1, int(wz > 0) + 2 * int(wxy > 0))
    loss = (wt * sums / counts).sum() / active
    np.testing.assert_allclose(loss, tv_golden[f"{key}/loss"], rtol=1e-5, atol=1e-7)


def _kp_names(kp_golden):
    return [c for c in golden_cases(kp_golden) if c != "border"]


def test_kplanes_forward_matches_grid_sample_reference(kp_golden):
    for name in _kp_names(kp_golden):
        g = {k: kp_golden[f"{name}/{k}"] for k in ("pts", "rotations", "plane")}
        out = oracle.kplanes_fwd(g["pts"], g["rotations"], g["plane"])
        # the reference's own forward tolerance against grid_sample (test_kplanes_tilted.py:68)
        np.testing.assert_allclose(out, kp_golden[f"{name}/out_f32"], rtol=1e-4, atol=5e-6)
        np.testing.assert_allclose(out, kp_golden[f"{name}/out_f64"], rtol=1e-4, atol=5e-6)


def test_kplanes_gradients_fp64_anchored(kp_golden):
    # test_kplanes_tilted.py:71-95: the oracle's error against the fp64 torch
    # gradients must be no worse than 2x torch's own fp32 error.
    for name in _kp_names(kp_golden):
        g = {k: kp_golden[f"{name}/{k}"] for k in ("pts", "rotations", "plane", "upstream")}
        got = oracle.kplanes_bwd(g["pts"], g["rotations"], g["plane"], g["upstream"])
        for label, mine in zip(("pts", "rotations", "plane"), got):
            ref64 = kp_golden[f"{name}/grad_{label}_f64"]
            err_torch = np.abs(kp_golden[f"{name}/grad_{label}_f32"].astype(np.float64) - ref64).max()
            err_oracle = np.abs(mine.astype(np.float64) - ref64).max()
            assert err_oracle <= max(2.0 * err_torch, 1e-6), (name, label, err_oracle, err_torch)


def test_kplanes_border_points(kp_golden):
    pts, rot, plane = (kp_golden[f"border/{k}"] for k in ("pts", "rotations", "plane"))
    out = oracle.kplanes_fwd(pts, rot, plane)
    np.testing.assert_allclose(out, kp_golden["border/out_f32"], rtol=1e-5, atol=1e-6)
    gp, _, _ = oracle.kplanes_bwd(pts, rot, plane, np.ones_like(out))
    np.testing.assert_allclose(gp, kp_golden["border/grad_pts_f32"], rtol=1e-4, atol=1e-6)


# ── four-tap K-Planes (reference_tv, test_kplanes_tilted.py:200-220) ─────────


def _kp_tv_names(kp_tv_golden):
    return [c for c in golden_cases(kp_tv_golden) if c != "tv_border"]


def test_kplanes_tv_forward_matches_reference_tv(kp_tv_golden):
    for name in _kp_tv_names(kp_tv_golden):
        g = {k: kp_tv_golden[f"{name}/{k}"] for k in ("pts", "rotations", "plane")}
        h = float(kp_tv_golden[f"{name}/h"])
        out = oracle.kplanes_tv_fwd(g["pts"], g["rotations"], g["plane"], h)
        assert out.shape == kp_tv_golden[f"{name}/out_f32"].shape
        # tap 0 is the base forward, bit for bit
        np.testing.assert_array_equal(out[0], oracle.kplanes_fwd(g["pts"], g["rotations"], g["plane"]))
        # the reference test's tolerance for all four taps (test_kplanes_tilted.py:246)
        np.testing.assert_allclose(out, kp_tv_golden[f"{name}/out_f32"], rtol=1e-4, atol=5e-6)
        np.testing.assert_allclose(out, kp_tv_golden[f"{name}/out_f64"], rtol=1e-4, atol=5e-6)


def test_kplanes_tv_gradients_fp64_anchored(kp_tv_golden):
    # test_kplanes_tilted.py:249-286: error against the fp64 torch gradients no
    # worse than K x torch's own fp32 error (K = 4 for rotations, 2 elsewhere).
    for name in _kp_tv_names(kp_tv_golden):
        g = {k: kp_tv_golden[f"{name}/{k}"] for k in ("pts", "rotations", "plane", "upstream")}
        h = float(kp_tv_golden[f"{name}/h"])
        got = oracle.kplanes_tv_bwd(g["pts"], g["rotations"], g["plane"], g["upstream"], h)
        for label, mine in zip(("pts", "rotations", "plane"), got):
            ref64 = kp_tv_golden[f"{name}/grad_{label}_f64"]
            err_torch = np.abs(kp_tv_golden[f"{name}/grad_{label}_f32"].astype(np.float64) - ref64).max()
            err_oracle = np.abs(mine.astype(np.float64) - ref64).max()
            k = 4.0 if label == "rotations" else 2.0
            assert err_oracle <= max(k * err_torch, 1e-6), (name, label, err_oracle, err_torch)


def test_kplanes_tv_border_points(kp_tv_golden):
    pts, rot, plane = (kp_tv_golden[f"tv_border/{k}"] for k in ("pts", "rotations", "plane"))
    h = float(kp_tv_golden["tv_border/h"])
    out = oracle.kplanes_tv_fwd(pts, rot, plane, h)
    np.testing.assert_allclose(out, kp_tv_golden["tv_border/out_f32"], rtol=1e-4, atol=1e-6)
    gp, _, _ = oracle.kplanes_tv_bwd(pts, rot, plane, np.ones_like(out), h)
    np.testing.assert_allclose(gp, kp_tv_golden["tv_border/grad_pts_f32"], rtol=1e-4, atol=1e-6)


def test_torch_restatement_matches_reference_definitions(tv_golden, kp_golden):
    """The pure-torch CPU restatement timed as a baseline by bench.py
    (oracle/torch_ref.py) gives the golden fp64 results of the reference's own
    torch definitions."""
    import torch

    from oracle import torch_ref

    for name in _tv_names(tv_golden):
        vol = torch.from_numpy(tv_golden[f"{name}/vol"]).double()
        iso_ref = tv_golden[f"{name}/iso_loss"]
        if not np.isnan(iso_ref):
            np.testing.assert_allclose(torch_ref.tv_iso(vol, 1e-8).item(), iso_ref, rtol=1e-10)
        np.testing.assert_allclose(torch_ref.tv_sq(vol).item(), tv_golden[f"{name}/sq_loss"], rtol=1e-10)
        np.testing.assert_allclose(torch_ref.tv_l1(vol).numpy(), tv_golden[f"{name}/l1_sums"], rtol=1e-10)
    names = sorted({k.split("/")[0] for k in kp_golden if not k.startswith("border")})
    for name in names:
        t = [torch.from_numpy(kp_golden[f"{name}/{k}"]).double() for k in ("pts", "rotations", "plane")]
        out = torch_ref.kplanes_tilted(*t).numpy()
        np.testing.assert_allclose(out, kp_golden[f"{name}/out_f64"], rtol=1e-10, atol=1e-12)
