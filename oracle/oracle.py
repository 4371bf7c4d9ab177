"""Python access to the CPU oracle (TEST INFRASTRUCTURE ONLY).

This module is the oracle: it wraps the C restatement of the
reference kernels (``tv_oracle.c``, ``kplanes_oracle.c``) and, when it has
been built, the reference's own ``_core`` extension compiled from its sources
into ``_ref/``. Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` import it; the product never does.

All arrays are numpy ``float32`` C-contiguous. Shapes follow the reference:
TV volumes ``[B, D, H, W]``; K-Planes ``pts [N, 3]``, ``R [T, 3, 3]``,
``plane [3T, C, H, W]`` (parameter layout), ``out [N, T*C]``.
"""

from __future__ import annotations

import ctypes
import importlib.util
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "build" / "liboracle_qc.so"
REF_CORE_PATH = HERE / "_ref" / ("_core" + sysconfig.get_config_var("EXT_SUFFIX"))

_lib = None
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)


def build() -> None:
    """Compiles the oracle library (gcc) if it is missing or stale."""
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    lib = ctypes.CDLL(str(LIB_PATH))
    i, f, L = ctypes.c_int, ctypes.c_float, ctypes.c_long
    sig = {
        "oracle_tv_iso_loss": [_f32p, i, i, i, i, f, _f64p],
        "oracle_tv_iso_grad": [_f32p, f, _f32p, i, i, i, i, f],
        "oracle_tv_sq_loss": [_f32p, i, i, i, i, _f64p],
        "oracle_tv_sq_grad": [_f32p, f, _f32p, i, i, i, i],
        "oracle_tv_l1_loss": [_f32p, i, i, i, i, _f64p],
        "oracle_tv_l1_grad": [_f32p, _f32p, _f32p, i, i, i, i],
        "oracle_kplanes_fwd": [_f32p, _f32p, _f32p, _f32p, L, i, i, i, i],
        "oracle_kplanes_bwd": [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, L, i, i, i, i],
        "oracle_kplanes_tv_fwd": [_f32p, _f32p, _f32p, _f32p, L, i, i, i, i, f],
        "oracle_kplanes_tv_bwd": [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, L, i, i, i, i, f],
        "oracle_set_threads": [i],
        "oracle_get_threads": [],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int if name == "oracle_get_threads" else None
    _lib = lib
    return lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def set_threads(n: int) -> int:
    """Sets the OpenMP thread count of the oracle; returns the count in effect."""
    lib = _load()
    lib.oracle_set_threads(int(n))
    return int(lib.oracle_get_threads())


def threads() -> int:
    return int(_load().oracle_get_threads())


# ── TV ──────────────────────────────────────────────────────────────────────


def _as4d(vol: np.ndarray) -> np.ndarray:
    v = _f32(vol)
    return v.reshape(-1, *v.shape[-3:])


def tv_iso_sum(vol, eps: float) -> float:
    """Σ over corners of sqrt(dd²+dh²+dw²+eps) (tv_loss.cu:47-96)."""
    v = _as4d(vol)
    out = np.zeros(1, np.float64)
    _load().oracle_tv_iso_loss(_p(v), *v.shape, float(eps), out.ctypes.data_as(_f64p))
    return float(out[0])


def tv_iso_loss(vol, eps: float) -> float:
    """Mean over corners, as the op returns (core/_ops.py:19-21, :119)."""
    v = _as4d(vol)
    b, d, h, w = v.shape
    return tv_iso_sum(v, eps) / max(1, b * (d - 1) * (h - 1) * (w - 1))


def tv_iso_grad(vol, g_scaled: float, eps: float) -> np.ndarray:
    v = _as4d(vol)
    out = np.empty_like(v)
    _load().oracle_tv_iso_grad(_p(v), float(g_scaled), _p(out), *v.shape, float(eps))
    return out.reshape(np.shape(vol))


def tv_sq_loss(vol) -> float:
    v = _as4d(vol)
    out = np.zeros(1, np.float64)
    _load().oracle_tv_sq_loss(_p(v), *v.shape, out.ctypes.data_as(_f64p))
    return float(out[0])


def tv_sq_grad(vol, g: float) -> np.ndarray:
    v = _as4d(vol)
    out = np.empty_like(v)
    _load().oracle_tv_sq_grad(_p(v), float(g), _p(out), *v.shape)
    return out.reshape(np.shape(vol))


def tv_l1_loss(vol) -> np.ndarray:
    v = _as4d(vol)
    out = np.zeros(3, np.float64)
    _load().oracle_tv_l1_loss(_p(v), *v.shape, out.ctypes.data_as(_f64p))
    return out


def tv_l1_grad(vol, g3) -> np.ndarray:
    v = _as4d(vol)
    g = _f32(np.asarray(g3).reshape(3))
    out = np.empty_like(v)
    _load().oracle_tv_l1_grad(_p(v), _p(g), _p(out), *v.shape)
    return out.reshape(np.shape(vol))


# ── K-Planes ────────────────────────────────────────────────────────────────


def kplanes_fwd(pts, R, plane) -> np.ndarray:
    p, r, g = _f32(pts), _f32(R), _f32(plane)
    n, t = p.shape[0], r.shape[0]
    c, h, w = g.shape[1:]
    out = np.empty((n, t * c), np.float32)
    _load().oracle_kplanes_fwd(_p(p), _p(r), _p(g), _p(out), n, t, c, h, w)
    return out


def kplanes_bwd(pts, R, plane, gout):
    """(grad_pts, grad_R, grad_plane) of Σ out·gout, plane in [3T, C, H, W]."""
    p, r, g, go = _f32(pts), _f32(R), _f32(plane), _f32(gout)
    n, t = p.shape[0], r.shape[0]
    c, h, w = g.shape[1:]
    gp = np.empty_like(p)
    gr = np.empty_like(r)
    gg = np.empty_like(g)
    _load().oracle_kplanes_bwd(_p(p), _p(r), _p(g), _p(go), _p(gp), _p(gr), _p(gg), n, t, c, h, w)
    return gp, gr, gg


def kplanes_tv_fwd(pts, R, plane, h: float) -> np.ndarray:
    """Four-tap form: out [4, N, T*C], tap k at R_t·p (+ h·R_t[:, k-1])."""
    p, r, g = _f32(pts), _f32(R), _f32(plane)
    n, t = p.shape[0], r.shape[0]
    c, hh, w = g.shape[1:]
    out = np.empty((4, n, t * c), np.float32)
    _load().oracle_kplanes_tv_fwd(_p(p), _p(r), _p(g), _p(out), n, t, c, hh, w, float(h))
    return out


def kplanes_tv_bwd(pts, R, plane, gout, h: float):
    """(grad_pts, grad_R, grad_plane) of Σ out·gout for the four-tap form."""
    p, r, g, go = _f32(pts), _f32(R), _f32(plane), _f32(gout)
    n, t = p.shape[0], r.shape[0]
    c, hh, w = g.shape[1:]
    gp = np.empty_like(p)
    gr = np.empty_like(r)
    gg = np.empty_like(g)
    _load().oracle_kplanes_tv_bwd(_p(p), _p(r), _p(g), _p(go), _p(gp), _p(gr), _p(gg), n, t, c, hh, w,
                                  float(h))
    return gp, gr, gg


# ── the reference's own CUDA `_core`, built from its sources ────────────────

_ref_core = None


def ref_core():
    """The reference's compiled ``_core`` module, or None when not built here."""
    global _ref_core
    if _ref_core is not None:
        return _ref_core
    if not REF_CORE_PATH.exists():
        return None
    spec = importlib.util.spec_from_file_location("qc_reference_build._core", REF_CORE_PATH)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    _ref_core = mod
    return mod


def available_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


__all__ = [
    "build",
    "set_threads",
    "threads",
    "tv_iso_sum",
    "tv_iso_loss",
    "tv_iso_grad",
    "tv_sq_loss",
    "tv_sq_grad",
    "tv_l1_loss",
    "tv_l1_grad",
    "kplanes_fwd",
    "kplanes_bwd",
    "kplanes_tv_fwd",
    "kplanes_tv_bwd",
    "ref_core",
    "available_cores",
]

if __name__ == "__main__":  # pragma: no cover
    build()
    print("oracle threads:", threads(), file=sys.stderr)
