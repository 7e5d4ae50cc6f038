"""Failure detection without a GPU fault: a bounded device-side wait that runs out.

jk_debug_window_stalled_producer runs the window kernel with a producer warp that issues
nothing, so the consumer warps' bounded mbarrier waits give up (about 2 s each, the same
bound every wait of every kernel has). The kernel then records JK_ERR_DEVICE_TIMEOUT in the
library's device error word, releases its TMEM and returns; the host reads the status with
jk_device_status, and a normal call right after on the same context still succeeds. Nothing
here faults, traps or hangs the GPU: the stall is a flag nothing sets, and every wait is
bounded."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import jakal_net_b200 as jk

    dev = torch.device("cuda", 0)
    lib = jk._LIBRARY
    status = ctypes.c_int(-99)
    assert lib.jk_device_status(None, ctypes.byref(status)) == 0  # clear any earlier word
    g = torch.Generator().manual_seed(0)
    B, N, D, R = 1, 128, 64, 64
    val = torch.randn(B, N, D, generator=g).to(dev, torch.bfloat16)
    state = torch.randn(B, N, generator=g).to(dev, torch.bfloat16)
    w = (torch.randn(R, D, generator=g) / D ** 0.5).to(dev, torch.bfloat16)
    pt = jk.lowrank_project(val, w)
    out_state = torch.full((B, N), 7.0, device=dev, dtype=torch.float32)
    out_val = torch.full((B, N, D), 7.0, device=dev, dtype=torch.float32)
    rc = lib.jk_debug_window_stalled_producer(pt.data_ptr(), pt.data_ptr(), B, N, N, pt.shape[-1], 1,
                                              state.data_ptr(), 1, val.data_ptr(), D, 16, out_state.data_ptr(),
                                              out_val.data_ptr(), 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0  # the launch itself is fine; the failure is reported by the device
    assert lib.jk_device_status(None, ctypes.byref(status)) == 0
    assert status.value == -6  # JK_ERR_DEVICE_TIMEOUT
    assert torch.count_nonzero(out_val) == 0  # the unwound kernel wrote zeros, no stale data
    # the context is intact: the error word was cleared and a normal launch works
    assert lib.jk_device_status(None, ctypes.byref(status)) == 0 and status.value == 0
    st, vv = jk.propagation_window("low_rank_bilinear", torch.ones(R, device=dev) / R ** 0.5, None, w, None, w,
                                   None, "softsign", val, state, val, 16, 128, 128)
    torch.cuda.synchronize()
    assert torch.isfinite(vv.float()).all() and vv.abs().sum() > 0
    assert lib.jk_device_status(None, ctypes.byref(status)) == 0 and status.value == 0
