"""GPU parity of the reference-facing ops (the native-module contract of jakal_net_b200)
against the CPU oracle, through the C ABI, on seeded bf16 inputs.

The oracle is evaluated on the same bf16 projections the library produced
(jk.lowrank_project), so the comparison isolates the fused kernels; outputs are bf16 like
the reference op returns them, hence the bf16 rounding step in the tolerance."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import parity

pytestmark = pytest.mark.gpu
OUT_RTOL = parity.VAL_RTOL + 2 ** -8  # kernel tolerance + one bf16 rounding of the output


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda", 0)


def _t(a, dev, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev).to(dtype)


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("compress", ["softsign", "signed_abs_softmax", "signed_entmax15"])
@pytest.mark.parametrize("k", [3, 32])
def test_propagation_topk_op(dev, compress, k):
    import jakal_net_b200 as jk

    g = np.random.default_rng(11 + k)
    B, N, D, R = 2, 333, 96, 64
    val = _t(g.standard_normal((B, N, D)), dev)
    state = _t(g.standard_normal((B, N)), dev)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _t(np.full(R, R ** -0.5), dev, torch.float32)
    bias = torch.tensor(0.05, device=dev)
    st, vv = jk.propagation_topk("low_rank_bilinear", core, bias, w_s, None, w_t, None, compress, val, state, val,
                                 k, 128, 128)
    assert st.dtype == torch.bfloat16 and vv.shape == val.shape
    pt = _np(jk.lowrank_project(val, w_t))
    ps = _np(jk.lowrank_project(val, w_s, core=core))
    o_st, o_val, _, _ = oracle.propagation_topk(pt, ps, _np(state), _np(val), k, bias=0.05, compress_name=compress)
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="state")


def test_propagation_window_topk_op_state_weighted(dev):
    # state_weight_edges folds softplus(state) into the projected inputs (propagation.py:165-174)
    import jakal_net_b200 as jk

    g = np.random.default_rng(5)
    B, N, D, R, W, k = 3, 700, 128, 64, 200, 16
    val = _t(g.standard_normal((B, N, D)), dev)
    state = _t(g.standard_normal((B, N)), dev)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _t(np.linspace(0.05, 0.2, R), dev)
    strength = torch.nn.functional.softplus(state.float())
    pstate = strength.to(torch.bfloat16)
    pval = (val.float() * strength[..., None]).to(torch.bfloat16)
    st, vv = jk.propagation_window_topk("low_rank_bilinear", core, None, w_s, None, w_t, None, "softsign", val,
                                        pstate, pval, W, k)
    pt = _np(jk.lowrank_project(val, w_t))
    ps = _np(jk.lowrank_project(val, w_s, core=core))
    o_st, o_val, _, _ = oracle.propagation_topk(pt, ps, _np(pstate), _np(pval), k, window=W)
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="state")


@pytest.mark.parametrize("temperature", [1.0, 0.5])
def test_transition_query_topk_op(dev, temperature):
    import jakal_net_b200 as jk

    g = np.random.default_rng(21)
    B, S, Q, D, R, k = 2, 1500, 200, 64, 64, 16
    src = _t(g.standard_normal((B, S, D)), dev)
    qv = _t(0.02 * g.standard_normal((B, Q, D)), dev)
    sstate = _t(g.standard_normal((B, S)), dev)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _t(np.ones(R), dev)
    bias = torch.tensor(0.3, device=dev)
    sender = torch.nn.functional.softplus(sstate.float()).to(torch.bfloat16)
    st, vv = jk.transition_query_topk("low_rank_bilinear_route", w_s, None, w_t, None, core, bias, None, None, None,
                                      None, temperature, sender, src, qv, sstate, src, k, 128, 128, True)
    sp = _np(jk.lowrank_project(src, w_s, core=core, temperature=temperature))
    qp = _np(jk.lowrank_project(qv, w_t))
    o_st, o_val, _, _ = oracle.transition_query_topk(qp, sp, _np(sstate), _np(src), _np(sender), k,
                                                     bias=0.3 / temperature)
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="state")


@pytest.mark.parametrize("compress", ["softmax", "signed_abs_softmax", "signed_entmax15"])
def test_transition_pairwise_topk_op(dev, compress):
    import jakal_net_b200 as jk

    g = np.random.default_rng(31)
    B, S, Dn, D, R, k = 2, 700, 150, 64, 64, 8
    src = _t(g.standard_normal((B, S, D)), dev)
    dst = _t(g.standard_normal((B, Dn, D)), dev)
    sstate = _t(g.standard_normal((B, S)), dev)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _t(np.ones(R), dev)
    sender = torch.nn.functional.softplus(sstate.float()).to(torch.bfloat16)
    st, vv = jk.transition_pairwise_topk("low_rank_bilinear_route", w_s, None, w_t, None, core, None, None, None,
                                         None, None, 1.0, sender, src, dst, sstate, src, k, 128, 128,
                                         route_compress_name=compress)
    sp = _np(jk.lowrank_project(src, w_s, core=core))
    dp = _np(jk.lowrank_project(dst, w_t))
    o_st, o_val = oracle.transition_pairwise_topk(sp, dp, _np(sstate), _np(src), _np(sender), k,
                                                  compress_name=compress)
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="state")


def test_device_status_is_clean_after_the_ops(dev):
    import ctypes

    import jakal_net_b200 as jk

    status = ctypes.c_int(-99)
    assert jk._LIBRARY.jk_device_status(None, ctypes.byref(status)) == 0
    assert status.value == 0


@pytest.mark.parametrize("compress", ["softsign", "signed_abs_softmax", "signed_entmax15"])
@pytest.mark.parametrize("shape", [(2, 300, 128, 40), (1, 700, 384, 512), (2, 256, 64, -1), (1, 1024, 512, 511)])
def test_window_and_dense_propagation_op(dev, compress, shape):
    import jakal_net_b200 as jk

    B, N, D, W = shape
    g = np.random.default_rng(N + D)
    R = 64
    val = _t(g.standard_normal((B, N, D)), dev)
    state = _t(g.standard_normal((B, N)), dev)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _t(np.full(R, R ** -0.5), dev)
    bias = torch.tensor(-0.1, device=dev)
    if W >= 0:
        st, vv = jk.propagation_window("low_rank_bilinear", core, bias, w_s, None, w_t, None, compress, val, state,
                                       val, W, 128, 128)
    else:
        st, vv = jk.propagation_dense("low_rank_bilinear", core, bias, w_s, None, w_t, None, compress, val, state,
                                      val, None, 128, 128)
    pt = _np(jk.lowrank_project(val, w_t))
    ps = _np(jk.lowrank_project(val, w_s, core=core))
    o_st, o_val = oracle.propagation_masked_dense(pt, ps, _np(state), _np(val), window=None if W < 0 else W,
                                                  bias=-0.1, compress_name=compress)
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="state")


def test_query_dense_propagation_op(dev):
    import jakal_net_b200 as jk

    g = np.random.default_rng(77)
    B, Q, S, D, R = 2, 130, 900, 192, 64
    qv = _t(g.standard_normal((B, Q, D)), dev)
    sv = _t(g.standard_normal((B, S, D)), dev)
    state = _t(g.standard_normal((B, S)), dev)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _t(np.full(R, R ** -0.5), dev)
    st, vv = jk.propagation_query_dense("low_rank_bilinear", core, None, w_s, None, w_t, None, "signed_abs_softmax",
                                        qv, sv, state, sv, 128, 128)
    pt = _np(jk.lowrank_project(qv, w_t))
    ps = _np(jk.lowrank_project(sv, w_s, core=core))
    o_st, o_val = oracle.propagation_masked_dense(pt, ps, _np(state), _np(sv), window=None,
                                                  compress_name="signed_abs_softmax")
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="state")


@pytest.mark.parametrize("compress", ["softmax", "signed_abs_softmax", "signed_entmax15"])
@pytest.mark.parametrize("shape", [(2, 700, 300, 128), (1, 130, 1000, 64)])
def test_transition_pairwise_dense_op(dev, compress, shape):
    import jakal_net_b200 as jk

    B, S, Dn, D = shape
    g = np.random.default_rng(S + Dn)
    R = 64
    src = _t(g.standard_normal((B, S, D)), dev)
    dst = _t(g.standard_normal((B, Dn, D)), dev)
    sstate = _t(g.standard_normal((B, S)), dev)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _t(np.ones(R), dev)
    sender = torch.nn.functional.softplus(sstate.float()).to(torch.bfloat16)
    st, vv = jk.transition_pairwise_dense("low_rank_bilinear_route", w_s, None, w_t, None, core,
                                          torch.tensor(0.1, device=dev), None, None, None, None, compress, 0.8,
                                          sender, src, dst, sstate, src, 128, 128)
    sp = _np(jk.lowrank_project(src, w_s, core=core, temperature=0.8))
    dp = _np(jk.lowrank_project(dst, w_t))
    o_st, o_val = oracle.transition_dense(sp, dp, _np(sstate), _np(src), _np(sender), bias=0.1 / 0.8,
                                          compress_name=compress)
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="state")


@pytest.mark.parametrize("D", [64, 128])
def test_diagonal_bilinear_topk_op(dev, D):
    # diagonal_bilinear (modules.py:37-53): score = target . (source * w_hat) + b
    import jakal_net_b200 as jk

    g = np.random.default_rng(D)
    B, N, k = 2, 400, 16
    val = _t(g.standard_normal((B, N, D)) / np.sqrt(D), dev)
    state = _t(g.standard_normal((B, N)), dev)
    w = np.abs(g.standard_normal(D)) + 0.5
    w_hat = _t(w * np.sqrt(D) / np.linalg.norm(w), dev)
    st, vv = jk.propagation_topk("diagonal_bilinear", w_hat, torch.tensor(0.02, device=dev), None, None, None, None,
                                 "signed_abs_softmax", val, state, val, k, 128, 128)
    v = _np(val)
    ps = oracle.round_to(v * _np(w_hat), "bf16")
    o_st, o_val, _, _ = oracle.topk_from_scores(oracle.lowrank_scores(v, ps), _np(state), v, k, bias=0.02,
                                                compress_name="signed_abs_softmax")
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="state")


@pytest.mark.parametrize("compress", ["softmax", "signed_abs_softmax"])
def test_transition_routes_form_is_deterministic_and_matches_the_scatter(dev, compress):
    """The per-source transition's routes form (dense route matrix from the fused kernel,
    then a GEMM) gives bit-identical results on repeated calls and agrees with the atomic
    scatter entry point (jk_transition_pairwise_topk_forward) within the kernel tolerance."""
    import jakal_net_b200 as jk

    g = np.random.default_rng(41)
    B, S, Dn, D, R, k = 2, 900, 130, 96, 64, 12
    src = _t(g.standard_normal((B, S, D)), dev)
    dst = _t(g.standard_normal((B, Dn, D)), dev)
    sstate = _t(g.standard_normal((B, S)), dev)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _t(np.ones(R), dev)
    sender = torch.nn.functional.softplus(sstate.float()).to(torch.bfloat16)
    args = ("low_rank_bilinear_route", w_s, None, w_t, None, core, None, None, None, None, None, 1.0, sender, src,
            dst, sstate, src, k, 128, 128)
    a = jk.transition_pairwise_topk(*args, route_compress_name=compress)
    b = jk.transition_pairwise_topk(*args, route_compress_name=compress)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    sp = jk.lowrank_project(src, w_s, core=core)
    dp = jk.lowrank_project(dst, w_t)
    accum = torch.empty(B * Dn * (D + 1) + 4, device=dev, dtype=torch.float32)
    st = torch.empty(B, Dn, device=dev, dtype=torch.float32)
    vv = torch.empty(B, Dn, D, device=dev, dtype=torch.float32)
    code = {"softmax": 3, "signed_abs_softmax": 1}[compress]
    rc = jk._LIBRARY.jk_transition_pairwise_topk_forward(
        sp.data_ptr(), dp.data_ptr(), B, S, Dn, sp.shape[-1], 1, sstate.data_ptr(), sender.data_ptr(), 1,
        src.data_ptr(), D, 1, k, 0.0, None, code, accum.data_ptr(), st.data_ptr(), vv.data_ptr(), 0,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    parity.assert_rows_close(_np(a[1]), _np(vv), rtol=OUT_RTOL, what="routes vs scatter val")
    parity.assert_rows_close(_np(a[0]), _np(st), rtol=OUT_RTOL, what="routes vs scatter state")


def test_split_stack_planes_and_route_aggregate(dev):
    """jk_split_stack_bf16 stacks hi / lo planes (with the extra column and zero padding) as
    asked, and the one-GEMM route aggregate of f32 values built on it matches an f64 aggregate
    of the same routes to the split's ~2^-16 relative accuracy."""
    import jakal_net_b200 as jk

    g = torch.Generator().manual_seed(11)
    B, S, C, Dn = 3, 37, 20, 9
    x = torch.randn(B, S, C, generator=g).to(dev)
    extra = torch.randn(B, S, generator=g).to(dev)
    out = jk._split_stack(x, extra, 24, (0, 1, 0))
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    e_hi = extra.to(torch.bfloat16)
    e_lo = (extra - e_hi.float()).to(torch.bfloat16)
    for blk, (pl, ex) in enumerate(((hi, e_hi), (lo, e_lo), (hi, e_hi))):
        part = out[:, blk * S:(blk + 1) * S]
        assert torch.equal(part[..., :C], pl)
        assert torch.equal(part[..., C], ex)
        assert not part[..., C + 1:].any()
    routes = torch.rand(B, S, Dn, generator=g).to(dev) * (torch.rand(B, S, Dn, generator=g) < 0.3).to(dev)
    st, vv = jk.routes_aggregate(routes, extra, x)
    want_v = torch.einsum("bsd,bsc->bdc", routes.double(), x.double())
    want_s = torch.einsum("bsd,bs->bd", routes.double(), extra.double())
    scale_v = want_v.abs() + want_v.pow(2).mean(dim=-1, keepdim=True).sqrt()
    assert ((vv.double() - want_v).abs() / scale_v).max().item() < 1e-4
    assert ((st.double() - want_s).abs() / (want_s.abs() + want_s.pow(2).mean().sqrt())).max().item() < 1e-4
