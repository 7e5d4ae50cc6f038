"""Parity against the reference backend itself: the reference's own CUDA extension
(native/jakal_net_native.cpp + native/jakal_net_native_cuda.cu, built unchanged for sm_100a by
baseline/build_reference_cuda.py) and this backend are called with the same positional
arguments (native_backend.py:5567-5643) on identical seeded bf16 inputs.

This pins the bf16 rounding chain of the reference's CUDA fast paths
(jakal_net_native.cpp:6236-6251 window, :6355-6389 top-k: projections rounded in bf16,
core weight multiplied in bf16, f32 dot, f32 aggregate, output cast to bf16) -- the chain
the CPU oracle restates. Tolerance: values / states within 2e-3 per element plus one bf16
output rounding; top-k rows whose score sets differ only at a tie (the reference's tie order
depends on its thread stride, jakal_net_native_cuda.cu:111-121) are at most 0.5% of rows and
are excluded."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import parity

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "baseline"))
import build_reference_cuda  # noqa: E402  (baseline/build_reference_cuda.py)

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not build_reference_cuda.available(),
                       reason="reference CUDA extension not built (python baseline/build_reference_cuda.py)"),
]
OUT_RTOL = parity.VAL_RTOL + 2 ** -8


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    mod = build_reference_cuda.load_built()
    assert "cuda" in mod.supported_devices()
    return mod


def _inputs(B, N, D, R, seed):
    g = torch.Generator().manual_seed(seed)
    to = dict(device="cuda", dtype=torch.bfloat16)
    val = torch.randn(B, N, D, generator=g).to(**to)
    state = torch.randn(B, N, generator=g).to(**to)
    w_s = (torch.randn(R, D, generator=g) / D ** 0.5).to(**to)
    w_t = (torch.randn(R, D, generator=g) / D ** 0.5).to(**to)
    core = (torch.rand(R, generator=g) + 0.5)
    core = (core / core.norm()).to(**to)
    bias = torch.tensor(0.05, device="cuda", dtype=torch.bfloat16)
    return val, state, w_s, w_t, core, bias


def _np(t):
    return t.detach().double().cpu().numpy()


def _rows_close_except_ties(got, want, max_frac=0.005, what=""):
    g, w = _np(got), _np(want)
    rms = np.sqrt(np.mean(w * w, axis=-1, keepdims=True))
    err = np.abs(g - w) / (np.abs(w) + rms + 1e-6)
    bad_rows = (err > OUT_RTOL).any(axis=-1) if g.ndim == 3 else (err > OUT_RTOL)
    assert bad_rows.mean() <= max_frac, f"{what}: {bad_rows.mean():.3%} of rows beyond tolerance"
    return bad_rows


# k = 64 is left out: on this B200 the reference's top-k kernel launch at k = 64 returns
# cudaErrorInvalidValue (a launch-configuration error of the reference build, not run again).
@pytest.mark.parametrize("k", [8, 32])
def test_propagation_topk_matches_reference_cuda(ref, k):
    import jakal_net_b200 as jk

    val, state, w_s, w_t, core, bias = _inputs(2, 700, 128, 64, 60 + k)
    args = ("low_rank_bilinear", core, bias, w_s, None, w_t, None, "softsign", val, state, val, k, 128, 128)
    want_state, want_val = ref.propagation_topk(*args)
    got_state, got_val = jk.propagation_topk(*args)
    assert got_val.dtype == want_val.dtype == torch.bfloat16
    bad = _rows_close_except_ties(got_val, want_val, what="val")
    g, w = _np(got_state), _np(want_state)
    rms = np.sqrt(np.mean(w * w, axis=-1, keepdims=True))
    err = (np.abs(g - w) / (np.abs(w) + rms))[~bad]
    assert err.max() <= OUT_RTOL


@pytest.mark.parametrize("window", [0, 37, 300])
def test_propagation_window_matches_reference_cuda(ref, window):
    import jakal_net_b200 as jk

    val, state, w_s, w_t, core, bias = _inputs(2, 600, 128, 64, 70 + window)
    args = ("low_rank_bilinear", core, bias, w_s, None, w_t, None, "softsign", val, state, val, window, 128, 128)
    want_state, want_val = ref.propagation_window(*args)
    got_state, got_val = jk.propagation_window(*args)
    assert got_val.dtype == want_val.dtype == torch.bfloat16
    parity.assert_rows_close(_np(got_val), _np(want_val), rtol=OUT_RTOL, what="window val")
    parity.assert_rows_close(_np(got_state), _np(want_state), rtol=OUT_RTOL, what="window state")
