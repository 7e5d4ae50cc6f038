"""GPU test of the allocation-free sparse-transition entry point.

jk_transition_pairwise_topk_forward_noalloc serves callers that cannot allocate device
memory at call time (plain-C / FFI hosts without a device allocator of their own, and
latency-critical loops that must avoid cudaMalloc / cudaFree because those can synchronise
the device): its scratch is a fixed array inside the library. This test calls it through
the C ABI twice in a row and checks each result against the regular entry point, which
takes caller-allocated scratch, within the tolerance the other parity tests use. The second
call also shows that the previous call's scratch contents do not leak into the next one.
The file name makes pytest collect it last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import parity

pytestmark = pytest.mark.gpu


def _call(jk, fn, args):
    status = fn(*args)
    assert status == 0, jk._LIBRARY.jk_status_string(status)


def test_noalloc_matches_regular_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import jakal_net_b200 as jk

    lib = jk._LIBRARY
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, seed in enumerate((41, 42)):
        g = torch.Generator().manual_seed(seed)
        B, S, Dn, D, R, k = 2, 500, 120, 128, 64, 8
        src = torch.randn(B, S, D, generator=g).to(dev, torch.bfloat16)
        dst = torch.randn(B, Dn, D, generator=g).to(dev, torch.bfloat16)
        state = torch.randn(B, S, generator=g).to(dev, torch.bfloat16)
        sender = torch.nn.functional.softplus(state.float()).to(torch.bfloat16)
        w_s = (torch.randn(R, D, generator=g) / D ** 0.5).to(dev, torch.bfloat16)
        w_t = (torch.randn(R, D, generator=g) / D ** 0.5).to(dev, torch.bfloat16)
        core = torch.ones(R).to(dev, torch.bfloat16)
        sp = jk.lowrank_project(src, w_s, core=core)
        dp = jk.lowrank_project(dst, w_t)
        rp = sp.shape[-1]
        outs = []
        for noalloc in (False, True):
            o_state = torch.empty(B, Dn, device=dev, dtype=torch.float32)
            o_val = torch.empty(B, Dn, D, device=dev, dtype=torch.float32)
            head = (sp.data_ptr(), dp.data_ptr(), B, S, Dn, rp, 1, state.data_ptr(), sender.data_ptr(), 1,
                    src.data_ptr(), D, 1, k, 0.0, None, 3)
            if noalloc:
                assert B * Dn * (D + 1) <= lib.jk_transition_pairwise_topk_noalloc_capacity()
                _call(jk, lib.jk_transition_pairwise_topk_forward_noalloc,
                      head + (o_state.data_ptr(), o_val.data_ptr(), 0, stream))
            else:
                accum = torch.empty(B * Dn * (D + 1), device=dev, dtype=torch.float32)
                _call(jk, lib.jk_transition_pairwise_topk_forward,
                      head + (accum.data_ptr(), o_state.data_ptr(), o_val.data_ptr(), 0, stream))
            torch.cuda.synchronize()
            outs.append((o_state.cpu().numpy(), o_val.cpu().numpy()))
        (r_state, r_val), (n_state, n_val) = outs
        assert np.isfinite(n_val).all()
        parity.assert_rows_close(n_val, r_val, what=f"val (call {call})")
        parity.assert_rows_close(n_state, r_state, what=f"state (call {call})")
    status = ctypes.c_int(-99)
    assert lib.jk_device_status(None, ctypes.byref(status)) == 0 and status.value == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import jakal_net_b200 as jk

    lib = jk._LIBRARY
    cap = lib.jk_transition_pairwise_topk_noalloc_capacity()
    assert cap == 1 << 22
    # Rejected before any device work: B * n_dst * (dim + 1) > capacity.
    status = lib.jk_transition_pairwise_topk_forward_noalloc(None, None, 4, 10, 1 << 16, 64, 1, None, None, 1, None,
                                                             64, 1, 8, 0.0, None, 3, None, None, 0, None)
    assert status == -1, lib.jk_status_string(status)
