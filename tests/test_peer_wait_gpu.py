"""A wait for another rank that is never answered gives up instead of hanging.

One GPU plays rank 0 of a two-rank D split whose rank 1 never runs: nothing
ever sets rank 1's flags. The halo exchange and the loss's cross-rank
reduction must each return after the configured bound, leave NaN in the loss,
set QC_FAULT_PEER_WAIT in the device fault word, and leave the context usable.
"""

from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT_NS = 50_000_000  # 50 ms


def test_unanswered_peer_waits_return_with_fault_bit():
    from quantem.cuda import _core
    from quantem.cuda._common import _workspace

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _core.device_fault_word(0, clear=True)
    B, Dp, H, W = 2, 6, 16, 32
    comm = [_core.peer_alloc(_core.tv_peer_comm_bytes()) for _ in range(2)]
    next_slab = _core.peer_alloc(B * 5 * H * W * 4)
    try:
        peers = _core.TvPeers(0, 2, TIMEOUT_NS, comm, 0, 0, next_slab, 5)
        slab = torch.rand((B, Dp, H, W), device=dev)
        grad = torch.empty_like(slab)
        acc = torch.zeros(1, device=dev)
        g = torch.ones(1, device=dev)
        ws = _workspace(dev)
        st = torch.cuda.current_stream().cuda_stream
        t0 = time.perf_counter()
        _core.tv_slab_halo_exchange_cuda(peers, 1, slab.data_ptr(), B, Dp, H, W, st)
        _core.tv_loss_3d_slab_peer_cuda(peers, 0, 1, _core.TV_SQ, _core.TV_LOSS | _core.TV_GRAD | _core.TV_ACC_OVERWRITE,
                                        slab.data_ptr(), g.data_ptr(), acc.data_ptr(), grad.data_ptr(),
                                        B, Dp, H, W, 1, Dp - 1, 0, 1, 0.0, 1.0, ws.data_ptr(), ws.numel(), st)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert torch.isnan(acc).all()
        assert _core.device_fault_word(0, clear=True) & _core.FAULT_PEER_WAIT
        assert elapsed < 5.0
        # the context still works
        x = torch.arange(8, device=dev, dtype=torch.float32)
        assert float(x.sum()) == 28.0
        assert _core.device_fault_word(0) == 0
    finally:
        torch.cuda.synchronize()
        for p in comm + [next_slab]:
            _core.peer_free(p)
