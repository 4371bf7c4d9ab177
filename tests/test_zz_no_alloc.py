"""The allocation-free isotropic TV entry point.

Some callers cannot call cudaMalloc where they compute the loss: applications
whose device memory is owned up front by one allocator or a fixed budget, and
hosts that allocate only at start-up. For them
`tv_loss_iso_3d_fwd_grad_noalloc_cuda` keeps the reduction scratch in a static
array inside the library instead of taking a caller workspace. This test
calls it through the C ABI on two calls in a row (new volumes each time, so
the second call runs over the first call's leftovers in the shared array) and
checks each result:

* bit for bit against the workspace entry point,
  `tv_loss_iso_3d_fwd_grad_cuda` (same sweep, same fixed-order reduction);
* against the CPU oracle, with the tolerances the other TV tests use
  (loss rel 1e-5, gradient rel 1e-4 of its largest magnitude);
* against the device's free memory as the driver reports it
  (`cudaMemGetInfo`, which sees every allocation in the process, not only
  torch's): a call after the first one on the device leaves it unchanged.

The file sorts last so that a run that stops at the first failure has run
every other test before it.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "quantem-cuda_b200" / "quantem" / "cuda" / "libquantem_cuda_b200.so"
FWD_RTOL = 1e-5
GRAD_RTOL = 1e-4
EPS = 1e-8


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
    g_up = 0.37
    g = torch.tensor([g_up], device="cuda")
    ws = torch.empty(lib.tv_loss_3d_workspace_bytes(B, D, H, W), dtype=torch.uint8, device="cuda")
    for call in range(2):
        vol_h = torch.rand(shape, generator=gen)
        vol = vol_h.cuda()
        acc_ref = torch.zeros(1, device="cuda")
        grad_ref = torch.empty_like(vol)
        assert lib.tv_loss_iso_3d_fwd_grad_cuda(vol.data_ptr(), g.data_ptr(), acc_ref.data_ptr(), grad_ref.data_ptr(),
                                                B, D, H, W, EPS, ws.data_ptr(), ws.numel(), st) == 0
        acc = torch.zeros(1, device="cuda")
        grad = torch.full_like(vol, float("nan"))
        torch.cuda.synchronize()
        free_before, _ = torch.cuda.mem_get_info()
        status = lib.tv_loss_iso_3d_fwd_grad_noalloc_cuda(vol.data_ptr(), g.data_ptr(), acc.data_ptr(),
                                                         grad.data_ptr(), B, D, H, W, EPS, st)
        assert status == 0, lib.quantem_cuda_last_error()
        torch.cuda.synchronize()
        free_after, _ = torch.cuda.mem_get_info()
        if call > 0:
            # the first call on a device may load the library's module; later
            # calls must not change the device's free memory at all
            assert free_after == free_before, (free_before, free_after)
        assert torch.equal(acc, acc_ref), (call, acc.item(), acc_ref.item())
        assert torch.equal(grad, grad_ref), f"gradient differs from the workspace entry, call {call}"
        x = vol_h.numpy()
        np.testing.assert_allclose(acc.item(), oracle.tv_iso_sum(x, EPS), rtol=FWD_RTOL)
        ref_grad = oracle.tv_iso_grad(x, g_up, EPS)
        err = np.abs(grad.cpu().numpy().astype(np.float64) - ref_grad).max()
        assert err <= GRAD_RTOL * np.abs(ref_grad).max(), (call, err)
