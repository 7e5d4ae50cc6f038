"""CPU-side tests: the C-ABI library loads and exports every declared symbol, the
native-module contract of jakal_net_b200, its argument checks (no compute without a GPU),
and the CPU port used as the benchmark baseline."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "jakal_b200.h"


def _declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\s*\*|int64_t|int)\s+(jk_\w+)\s*\(", text, re.M)))


def test_header_declares_the_entry_points():
    names = _declared_symbols()
    for expected in ("jk_lowrank_project", "jk_propagation_topk_forward", "jk_transition_query_topk_forward",
                     "jk_transition_pairwise_topk_forward", "jk_status_string", "jk_device_check",
                     "jk_device_status", "jk_padded_rank"):
        assert expected in names


def test_library_exports_every_declared_symbol():
    from jakal_net_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    # the ctypes binding knows every declared symbol too
    assert set(_declared_symbols()) <= set(_lib.SIGNATURES)


def test_status_strings_and_pure_helpers():
    import jakal_net_b200 as jk

    lib = jk._LIBRARY
    assert lib.jk_status_string(0) == b"ok"
    assert b"sm_100" in lib.jk_status_string(-4)
    assert lib.jk_padded_rank(1) == 64 and lib.jk_padded_rank(64) == 64 and lib.jk_padded_rank(65) == 128


def test_device_check_without_gpu_is_an_error_not_a_fallback():
    import jakal_net_b200 as jk

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert jk._LIBRARY.jk_device_check() == -4


def test_native_module_contract():
    import jakal_net_b200 as jk

    assert jk.backend_name() == "b200_sm100a"
    assert jk.supported_devices() == ["cuda"]
    ops = jk.supported_ops()
    assert "propagation_topk" in ops and "transition_query_topk" in ops and "transition_pairwise_topk" in ops
    # every advertised op is a callable of the module (the loader calls them by name)
    assert all(callable(getattr(jk, op, None)) for op in ops)
    # the training entry points of the autograd routes (native_backend.py:659-667, 5962-5975,
    # 5512-5612); the entmax window route needs the reference's own torch ops and stays off
    assert {"low_rank_pairwise_topk_forward_cuda", "low_rank_pairwise_topk_backward_cuda",
            "query_topk_reduce_backward_cuda", "softsign_backward_cuda", "softmax_backward_cuda",
            "low_rank_propagation_topk_forward_cuda", "low_rank_propagation_window_forward_cuda"} <= set(ops)
    assert "low_rank_propagation_window_entmax15_forward_cuda" not in ops


def test_cpu_tensors_raise_instead_of_falling_back():
    import jakal_net_b200 as jk

    val = torch.randn(1, 8, 16)
    w = torch.randn(4, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        jk.propagation_topk("low_rank_bilinear", torch.ones(4), None, w, None, w, None, "softsign", val,
                            torch.randn(1, 8), val, 2, 128, 128)


def test_unsupported_kind_and_compressor_are_rejected_before_any_launch():
    import jakal_net_b200 as jk

    with pytest.raises(RuntimeError, match="edge_compress_name"):
        jk.propagation_topk("low_rank_bilinear", None, None, None, None, None, None, "relu", None, None, None, 2, 1, 1)
    with pytest.raises(TypeError):
        jk._route_projections("mlp_route", None, None, None, None, None, None, None, None, None, None, 1.0, None, None)


def test_c_abi_rejects_bad_arguments_without_a_device():
    import jakal_net_b200 as jk

    lib = jk._LIBRARY
    # null pointers / bad k / bad dtype are caught before the device probe
    assert lib.jk_propagation_topk_forward(None, None, 1, 1, 1, 64, 1, None, None, 1, None, 8, 1, 4, -1, 0.0, None,
                                           0, None, None, 1, None, None, None) == -7
    buf = (ctypes.c_char * 64)()
    p = ctypes.addressof(buf)
    p16 = (p + 15) & ~15
    assert lib.jk_propagation_topk_forward(p16, p16, 1, 1, 1, 64, 1, p16, None, 1, p16, 8, 1, 65, -1, 0.0, None,
                                           0, p16, p16, 1, None, None, None) == -7
    assert lib.jk_propagation_topk_forward(p16, p16, 1, 1, 1, 64, 0, p16, None, 1, p16, 8, 1, 4, -1, 0.0, None,
                                           0, p16, p16, 1, None, None, None) == -2
    assert lib.jk_lowrank_project(p16, 4, 12, p16, 4, None, 1.0, 1, p16, 64, None) == -1  # dim % 8


def test_cpu_port_matches_oracle():
    import oracle
    from oracle import cpu_port

    g = np.random.default_rng(3)
    B, N, D, R, k, W = 2, 300, 24, 16, 8, 40
    pt = g.standard_normal((B, N, R)).astype(np.float32)
    ps = g.standard_normal((B, N, R)).astype(np.float32)
    st = g.standard_normal((B, N)).astype(np.float32)
    val = g.standard_normal((B, N, D)).astype(np.float32)
    for window in (W, None):
        o_st, o_val, _, _ = oracle.propagation_topk(pt, ps, st, val, k, window=window)
        c_st, c_val = cpu_port.window_topk_propagation(torch.from_numpy(pt), torch.from_numpy(ps),
                                                       torch.from_numpy(st), torch.from_numpy(val), k, window)
        np.testing.assert_allclose(c_st.numpy(), o_st, rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(c_val.numpy(), o_val, rtol=1e-4, atol=1e-4)


def test_bench_pair_count():
    import bench

    assert bench.pairs_per_batch_item(4, 2) == 1 + 2 + 3 + 3
    assert bench.PAIRS_PER_STEP == 8 * (513 * 2048 - 512 * 513 // 2)
