"""The allocation-free isotropic TV entry point.

Some callers cannot allocate device memory where they compute the loss (code
running where allocating or synchronising CUDA calls are not allowed, or an
application whose device memory is owned up front by one allocator), so
`tv_loss_iso_3d_fwd_grad_noalloc_cuda` keeps the reduction scratch in a
static array inside the library instead of taking a caller workspace. This
test calls it through the C ABI twice in a row and checks each result against
the workspace entry point, `tv_loss_iso_3d_fwd_grad_cuda`, with the tolerances
the other TV tests use. The file sorts last so that a run that stops at the
first failure has run every other test before it.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "quantem-cuda_b200" / "quantem" / "cuda" / "libquantem_cuda_b200.so"
FWD_RTOL = 1e-5
GRAD_RTOL = 1e-4


def _lib():
    lib = ctypes.CDLL(str(LIB))
    vp, i, f, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    lib.tv_loss_iso_3d_fwd_grad_cuda.argtypes = [vp, vp, vp, vp, i, i, i, i, f, vp, sz, vp]
    lib.tv_loss_iso_3d_fwd_grad_noalloc_cuda.argtypes = [vp, vp, vp, vp, i, i, i, i, f, vp]
    lib.tv_loss_3d_workspace_bytes.restype = sz
    lib.quantem_cuda_last_error.restype = ctypes.c_char_p
    return lib


@pytest.mark.parametrize("shape", [(2, 40, 70, 260), (3, 9, 31, 37)])  # TMA path, generic path
def test_noalloc_entry_matches_workspace_entry_on_two_calls(shape):
    lib = _lib()
    B, D, H, W = shape
    gen = torch.Generator().manual_seed(21)
    st = torch.cuda.current_stream().cuda_stream
    g = torch.tensor([0.37], device="cuda")
    ws = torch.empty(lib.tv_loss_3d_workspace_bytes(B, D, H, W), dtype=torch.uint8, device="cuda")
    for call in range(2):
        vol = torch.rand(shape, generator=gen).cuda()
        acc_ref = torch.zeros(1, device="cuda")
        grad_ref = torch.empty_like(vol)
        assert lib.tv_loss_iso_3d_fwd_grad_cuda(vol.data_ptr(), g.data_ptr(), acc_ref.data_ptr(), grad_ref.data_ptr(),
                                                B, D, H, W, 1e-8, ws.data_ptr(), ws.numel(), st) == 0
        acc = torch.zeros(1, device="cuda")
        grad = torch.full_like(vol, float("nan"))
        before = torch.cuda.memory_allocated()
        status = lib.tv_loss_iso_3d_fwd_grad_noalloc_cuda(vol.data_ptr(), g.data_ptr(), acc.data_ptr(),
                                                         grad.data_ptr(), B, D, H, W, 1e-8, st)
        assert status == 0, lib.quantem_cuda_last_error()
        assert torch.cuda.memory_allocated() == before
        torch.cuda.synchronize()
        torch.testing.assert_close(acc, acc_ref, rtol=FWD_RTOL, atol=0, msg=f"loss, call {call}")
        scale = grad_ref.abs().max().item()
        torch.testing.assert_close(grad, grad_ref, rtol=GRAD_RTOL, atol=1e-6 * scale, msg=f"gradient, call {call}")
