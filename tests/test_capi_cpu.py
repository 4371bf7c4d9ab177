"""CPU-only checks of the product boundary: the C-ABI library loads and
exports every entry point declared in include/*.h, the torch-free `_core`
binding carries the reference's function names, and the host-side argument
checks return status codes (no device work is issued)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
HEADERS = sorted((REPO / "include").glob("*.h"))
LIB = REPO / "quantem-cuda_b200" / "quantem" / "cuda" / "libquantem_cuda_b200.so"


def declared_functions() -> list[str]:
    names = []
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"#.*", "", text)
        names += re.findall(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", text)
    skip = {"extern", "if", "sizeof"}
    return sorted({n for n in names if n not in skip})


def test_header_declares_the_hot_path():
    names = declared_functions()
    for required in (
        "tv_loss_iso_3d_cuda",
        "tv_loss_iso_3d_grad_cuda",
        "tv_loss_sq_3d_cuda",
        "tv_loss_sq_3d_grad_cuda",
        "tv_loss_l1_3d_cuda",
        "tv_loss_l1_3d_grad_cuda",
        "kplanes_tilted_fuse_cuda",
        "kplanes_tilted_fuse_grad_cuda",
    ):
        assert required in names


DEBUG_LIB = LIB.with_name("libquantem_cuda_b200_debug.so")


@pytest.mark.parametrize("path", [LIB, DEBUG_LIB], ids=["release", "bounds-checked"])
def test_library_exports_every_declared_symbol(path):
    if not path.exists():
        pytest.skip(f"{path.name} not built")
    lib = ctypes.CDLL(str(path))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_status_strings_and_version():
    lib = ctypes.CDLL(str(LIB))
    lib.quantem_cuda_status_string.restype = ctypes.c_char_p
    assert lib.quantem_cuda_status_string(0) == b"QC_OK"
    assert lib.quantem_cuda_status_string(10001) == b"QC_ERR_INVALID_ARGUMENT"
    assert lib.quantem_cuda_cudart_version() >= 12000


def test_argument_errors_need_no_device():
    lib = ctypes.CDLL(str(LIB))
    lib.quantem_cuda_last_error.restype = ctypes.c_char_p
    f = lib.tv_loss_3d_slab_cuda
    f.restype = ctypes.c_int
    vp = ctypes.c_void_p
    i = ctypes.c_int
    fl = ctypes.c_float
    f.argtypes = [i, i, vp, vp, vp, vp, i, i, i, i, i, i, i, i, fl, fl, vp, ctypes.c_size_t, vp]
    # unknown variant
    assert f(7, 1, None, None, None, None, 1, 4, 4, 4, 0, 4, 0, 0, 0.0, 1.0, None, 0, None) == 10001
    assert b"variant" in lib.quantem_cuda_last_error()
    # the reference-signature loss entries need no workspace, but check their shape
    r = lib.tv_loss_sq_3d_cuda
    r.restype = ctypes.c_int
    r.argtypes = [vp, vp, i, i, i, i, vp]
    assert r(vp(16), vp(16), -1, 4, 4, 4, None) == 10001
    # the multi-level K-Planes entries check their level tables before any CUDA call
    lv = lib.kplanes_tilted_fuse_levels_cuda
    lv.restype = ctypes.c_int
    lv.argtypes = [vp, vp, i, ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(i), ctypes.POINTER(i),
                   ctypes.c_long, i, i, vp]
    grids = (vp * 9)(*([16] * 9))
    hs = (i * 9)(*([8] * 9))
    assert lv(vp(16), vp(16), 0, grids, grids, hs, hs, 4, 2, 8, None) == 10001
    assert lv(vp(16), vp(16), 9, grids, grids, hs, hs, 4, 2, 8, None) == 10001
    assert b"levels" in lib.quantem_cuda_last_error()
    assert lv(vp(16), vp(16), 2, None, grids, hs, hs, 4, 2, 8, None) == 10001
    big = (i * 2)(1 << 16, 1 << 16)
    assert lv(vp(16), vp(16), 2, grids, grids, big, big, 4, 2, 8, None) == 10001  # C*H*W >= 2^31
    # a mixed sweep needs two or three terms
    mx = lib.tv_loss_mix_3d_fwd_grad_cuda
    mx.restype = ctypes.c_int
    mx.argtypes = [i, i, vp, vp, vp, vp, i, i, i, i, fl, fl, vp, ctypes.c_size_t, vp]
    assert mx(2, 0, vp(16), vp(16), vp(16), vp(16), 1, 4, 4, 4, 1e-8, 1.0, vp(16), 1 << 20, None) == 10001
    assert b"two or three" in lib.quantem_cuda_last_error()
    # the allocation-free entry refuses shapes beyond the largest volume before any CUDA call
    na = lib.tv_loss_iso_3d_fwd_grad_noalloc_cuda
    na.restype = ctypes.c_int
    na.argtypes = [vp, vp, vp, vp, i, i, i, i, fl, vp]
    assert na(vp(16), vp(16), vp(16), vp(16), 1, 4, 1 << 16, 1 << 15, 1e-8, None) == 10001
    assert b"exceeds the largest volume" in lib.quantem_cuda_last_error()
    # loss without a workspace
    st = f(0, 1, vp(16), None, vp(16), None, 1, 4, 4, 4, 0, 4, 0, 0, 0.0, 1.0, None, 0, None)
    assert st == 10002
    # owned range outside the volume
    assert f(0, 2, vp(16), vp(16), None, vp(16), 1, 4, 4, 4, 0, 5, 0, 0, 0.0, 1.0, None, 0, None) == 10001
    k = lib.kplanes_tilted_fuse_cuda
    k.restype = ctypes.c_int
    k.argtypes = [vp, vp, vp, vp, ctypes.c_long, i, i, i, i, vp]
    assert k(vp(16), vp(16), vp(16), vp(16), 8, 2, 1 << 16, 1 << 8, 1 << 8, None) == 10001  # C*H*W >= 2^31


def test_core_binding_has_reference_names():
    from quantem.cuda import _core

    for name in (
        "tv_loss_iso_3d_cuda",
        "tv_loss_iso_3d_grad_cuda",
        "tv_loss_sq_3d_cuda",
        "tv_loss_sq_3d_grad_cuda",
        "tv_loss_l1_3d_cuda",
        "tv_loss_l1_3d_grad_cuda",
        "kplanes_tilted_fuse_cuda",
        "kplanes_tilted_fuse_grad_cuda",
    ):
        assert callable(getattr(_core, name))
    assert int(_core.__cudart_version__) >= 12000
    with pytest.raises(RuntimeError, match="QC_ERR_INVALID_ARGUMENT"):
        _core.tv_loss_3d_slab_cuda(9, 1, 0, 0, 0, 0, 1, 2, 2, 2, 0, 2, 0, 0, 0.0, 1.0, 0, 0, 0)


def _signature(fn) -> list[tuple[str, str]]:
    """(argument name, Python type) pairs from a pybind11 function's docstring."""
    head = fn.__doc__.strip().splitlines()[0]
    args = head[head.index("(") + 1 : head.rindex(")")]
    out = []
    for part in re.split(r",\s*(?=[A-Za-z_]+:)", args):
        name, typ = part.split(":", 1)
        out.append((name.strip(), "float" if "Float" in typ else "int"))
    return out


def test_core_binding_takes_the_reference_arguments():
    """Every function of the reference's `_core` (built from its sources into
    oracle/_ref/ when the reference tree was present; csrc/bindings/core.cpp:101-148,
    csrc/bindings/core/ml.cpp:89-128) exists here with the same argument names,
    order and kinds, so the reference's op layer calls this binding unchanged."""
    from oracle import oracle
    from quantem.cuda import _core

    ref = oracle.ref_core()
    if ref is None:
        pytest.skip("reference _core not built into oracle/_ref")
    names = [n for n in dir(ref) if n.endswith("_cuda")]
    assert len(names) == 10
    for name in names:
        assert _signature(getattr(_core, name)) == _signature(getattr(ref, name)), name


def test_peer_entries_reject_bad_arguments_without_a_device():
    from quantem.cuda import _core

    with pytest.raises(ValueError):
        _core.TvPeers(0, _core.MAX_PEER_RANKS + 1, 0, [1] * (_core.MAX_PEER_RANKS + 1), 0, 0, 0, 0)
    with pytest.raises(ValueError):
        _core.TvPeers(0, 2, 0, [1], 0, 0, 0, 0)  # one block per rank
    good = _core.TvPeers(0, 2, 0, [16, 32], 0, 0, 64, 5)
    with pytest.raises(RuntimeError, match="seq starts at 1"):
        _core.tv_slab_halo_exchange_cuda(good, 0, 128, 1, 5, 4, 4, 0)
    with pytest.raises(RuntimeError, match="null communication block"):
        _core.tv_slab_halo_exchange_cuda(_core.TvPeers(0, 2, 0, [16, 0], 0, 0, 64, 5), 1, 128, 1, 5, 4, 4, 0)
    with pytest.raises(RuntimeError, match="rank 2 outside"):
        _core.tv_slab_halo_exchange_cuda(_core.TvPeers(2, 2, 0, [16, 32], 0, 0, 0, 0), 1, 128, 1, 5, 4, 4, 0)
    with pytest.raises(RuntimeError, match="rank\\+1's slab missing"):
        _core.tv_slab_halo_exchange_cuda(_core.TvPeers(0, 2, 0, [16, 32], 0, 0, 0, 0), 1, 128, 1, 5, 4, 4, 0)
    with pytest.raises(RuntimeError, match="must include QC_TV_LOSS"):
        _core.tv_loss_3d_slab_peer_cuda(good, 0, 1, _core.TV_SQ, _core.TV_GRAD, 128, 0, 0, 256, 1, 5, 4, 4, 1, 4,
                                        0, 1, 0.0, 1.0, 0, 0, 0)
    with pytest.raises(RuntimeError, match="needs the slab layout"):
        _core.tv_loss_3d_slab_peer_cuda(good, 1, 1, _core.TV_SQ, _core.TV_LOSS, 128, 0, 0, 256, 1, 5, 4, 4, 0, 4,
                                        0, 1, 0.0, 1.0, 0, 0, 0)
    assert _core.tv_peer_comm_bytes() >= 8 * 2 * 4 * 8
    grp = _core.PeerGroup(0, 2, 0, [16, 32], [64, 128])
    with pytest.raises(RuntimeError, match="seq starts at 1"):
        _core.peer_allreduce_sum_f32_range_cuda(grp, 0, 0, 4, 0, 0)
    with pytest.raises(RuntimeError, match="negative offset, size or CTA count"):
        _core.peer_allreduce_sum_f32_range_cuda(grp, 1, -1, 4, 0, 0)
    with pytest.raises(RuntimeError, match="negative offset, size or CTA count"):
        _core.peer_allreduce_sum_f32_range_cuda(grp, 1, 0, 4, -2, 0)
