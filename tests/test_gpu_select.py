"""GPU parity of the select-aggregate kernel (jk_select_aggregate_forward): the path for every
shape the fused kernels do not take -- k > 64, f32 projections of rank > 32, scorers wider
than 128, projection dims that are not a multiple of 8 -- against the CPU oracle.

The reference takes any k through its blocked path (jakal_net_native.cpp:6390-6447,
6916-7087, 7089-7246); its CUDA kernels stop at k <= 64 (jakal_net_native_cuda.cu:2432-2434).
Tolerances: top-k index sets identical except ties within 1e-5 relative of the k-th score;
values / states within 2e-3 of the row's magnitude (f32 outputs: the kernel tolerance
alone; bf16 outputs: plus one bf16 rounding step)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import parity

pytestmark = pytest.mark.gpu
F32_RTOL = parity.VAL_RTOL
BF16_RTOL = parity.VAL_RTOL + 2 ** -8


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda", 0)


def _t(a, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev).to(dtype)


def _np(t):
    return t.detach().double().cpu().numpy()


def _check_selection(gpu_idx, ora_idx, ora_scores, full_scores):
    parity.set_full_scores(full_scores)
    return parity.tie_rows(gpu_idx, ora_idx, ora_scores)


@pytest.mark.parametrize("compress", ["softsign", "signed_abs_softmax", "signed_entmax15", "softmax"])
@pytest.mark.parametrize("k,window", [(65, -1), (128, 300), (256, -1), (999, 40)])
def test_select_aggregate_gather_matches_oracle(dev, compress, k, window):
    import jakal_net_b200 as jk

    g = np.random.default_rng(100 + k)
    B, T, S, R, D = 2, 300, 300, 48, 40
    row = _t(g.standard_normal((B, T, R)), dev)
    col = _t(g.standard_normal((B, S, R)) / np.sqrt(R), dev)
    state = _t(g.standard_normal((B, S)), dev)
    val = _t(g.standard_normal((B, S, D)), dev)
    bias = torch.tensor(0.1, device=dev)
    code = {"softsign": 0, "signed_abs_softmax": 1, "signed_entmax15": 2, "softmax": 3}[compress]
    st, vv, ss, ix = jk.select_aggregate(row, col, state, val, k, window=window, compress=code, bias=bias,
                                         return_selection=True)
    torch.cuda.synchronize()
    scores = oracle.lowrank_scores(_np(row), _np(col), 0.0)
    o_st, o_val, o_sc, o_ix = oracle.topk_from_scores(scores, _np(state), _np(val), min(k, S),
                                                      window=None if window < 0 else window, bias=0.1,
                                                      compress_name=compress)
    skip = _check_selection(ix.cpu().numpy(), o_ix, o_sc, scores + 0.1)
    assert skip.mean() < 0.05
    parity.assert_rows_close(_np(vv), o_val, skip_rows=skip, rtol=F32_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, skip_rows=skip, rtol=F32_RTOL, what="state")
    # the selection is returned in ascending column order
    gi = ix.cpu().numpy()
    for b in range(B):
        for t in range(0, T, 37):
            row_i = gi[b, t][gi[b, t] >= 0]
            assert (np.diff(row_i) > 0).all()


@pytest.mark.parametrize("compress", ["softmax", "signed_abs_softmax", "signed_entmax15"])
def test_select_aggregate_scatter_matches_oracle(dev, compress):
    import jakal_net_b200 as jk

    g = np.random.default_rng(7)
    B, S, Dn, R, D, k = 2, 500, 200, 32, 72, 100
    src = _t(g.standard_normal((B, S, R)), dev)
    dst = _t(g.standard_normal((B, Dn, R)) / np.sqrt(R), dev)
    state = _t(g.standard_normal((B, S)), dev)
    val = _t(g.standard_normal((B, S, D)), dev)
    sender = torch.nn.functional.softplus(state)
    code = {"signed_abs_softmax": 1, "signed_entmax15": 2, "softmax": 3}[compress]
    st, vv = jk.select_aggregate(src, dst, state, val, k, compress=code, sender=sender, scatter=True)
    o_st, o_val = oracle.transition_pairwise_topk(_np(src), _np(dst), _np(state), _np(val), _np(sender), k,
                                                  compress_name=compress)
    parity.assert_rows_close(_np(vv), o_val, rtol=F32_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=F32_RTOL, what="state")


def test_select_aggregate_blocks_agree_with_one_block(dev):
    """Row blocks of the materialised scores (a small score budget) give the same result
    as one block: the blocking is invisible."""
    import jakal_net_b200 as jk

    g = np.random.default_rng(8)
    B, T, R, D, k = 3, 257, 16, 24, 70
    row = _t(g.standard_normal((B, T, R)), dev)
    state = _t(g.standard_normal((B, T)), dev)
    val = _t(g.standard_normal((B, T, D)), dev)
    one = jk.select_aggregate(row, row, state, val, k, window=100)
    many = jk.select_aggregate(row, row, state, val, k, window=100, budget=B * (T + 3 * k) * 5)
    for a, b in zip(one, many):
        assert torch.equal(a, b)


@pytest.mark.parametrize("k", [65, 128, 256])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_propagation_topk_op_large_k(dev, k, dtype):
    """The reference-facing op with k > 64 (bf16: rank-64 projections; f32: rank 64 > 32)."""
    import jakal_net_b200 as jk

    g = np.random.default_rng(200 + k)
    B, N, D, R = 2, 400, 96, 64
    val = _t(g.standard_normal((B, N, D)), dev, dtype)
    state = _t(g.standard_normal((B, N)), dev, dtype)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev, dtype)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev, dtype)
    core = _t(np.full(R, R ** -0.5), dev)
    st, vv = jk.propagation_topk("low_rank_bilinear", core, None, w_s, None, w_t, None, "signed_abs_softmax",
                                 val, state, val, k, 128, 128)
    assert st.dtype == dtype and vv.shape == val.shape
    # the oracle on the reference's projections in the input dtype
    pt = (val @ w_t.t()).double().cpu().numpy()
    ps = ((val @ w_s.t()) * core.to(dtype)).double().cpu().numpy()
    scores = oracle.lowrank_scores(pt, ps, 0.0)
    o_st, o_val, o_sc, o_ix = oracle.topk_from_scores(scores, _np(state), _np(val), k,
                                                      compress_name="signed_abs_softmax")
    rtol = F32_RTOL if dtype == torch.float32 else BF16_RTOL
    parity.assert_rows_close(_np(vv), o_val, rtol=rtol, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=rtol, what="state")


def test_f32_rank64_window_and_odd_dims(dev):
    """f32 rank 64 (beyond the three-plane fused form) on the window op, and a projection dim
    of 5 (not a multiple of 8) on the fused bf16 top-k op."""
    import jakal_net_b200 as jk

    g = np.random.default_rng(9)
    B, N, D, R, W = 2, 260, 64, 64, 50
    val = _t(g.standard_normal((B, N, D)), dev)
    state = _t(g.standard_normal((B, N)), dev)
    w_s = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _t(np.full(R, R ** -0.5), dev)
    st, vv = jk.propagation_window("low_rank_bilinear", core, None, w_s, None, w_t, None, "softsign", val, state,
                                   val, W, 128, 128)
    pt = _np(val @ w_t.t())
    ps = _np((val @ w_s.t()) * core)
    o_st, o_val = oracle.propagation_masked_dense(pt, ps, _np(state), _np(val), window=W)
    parity.assert_rows_close(_np(vv), o_val, rtol=F32_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=F32_RTOL, what="state")

    D5 = 5
    val5 = _t(g.standard_normal((B, 90, D5)), dev, torch.bfloat16)
    w5s = _t(g.standard_normal((3, D5)), dev, torch.bfloat16)
    w5t = _t(g.standard_normal((3, D5)), dev, torch.bfloat16)
    c5 = _t(np.ones(3) / np.sqrt(3), dev)
    st5, vv5 = jk.propagation_topk("low_rank_bilinear", c5, None, w5s, None, w5t, None, "softsign", val5,
                                   val5[..., 0], val5, 4, 128, 128)
    pt5 = _np(val5 @ w5t.t())
    ps5 = _np((val5 @ w5s.t()) * c5.to(torch.bfloat16))
    o_st5, o_val5, o_sc5, o_ix5 = oracle.propagation_topk(pt5, ps5, _np(val5[..., 0]), _np(val5), 4)
    parity.assert_rows_close(_np(vv5), o_val5, rtol=BF16_RTOL, what="val dim 5")


def test_wide_diagonal_scorer_and_large_k_transitions(dev):
    """A diagonal scorer of dim 200 (> 128) on the dense op, and both transitions with k > 64."""
    import jakal_net_b200 as jk

    g = np.random.default_rng(10)
    B, N, D = 2, 150, 200
    val = _t(g.standard_normal((B, N, D)) / np.sqrt(D), dev)
    state = _t(g.standard_normal((B, N)), dev)
    w = _t(np.abs(g.standard_normal(D)) / np.sqrt(D), dev)
    st, vv = jk.propagation_dense("diagonal_bilinear", w, None, None, None, None, None, "signed_entmax15", val,
                                  state, val, None, 128, 128)
    ps = _np(val * w)
    o_st, o_val = oracle.propagation_masked_dense(_np(val), ps, _np(state), _np(val), window=None,
                                                  compress_name="signed_entmax15")
    parity.assert_rows_close(_np(vv), o_val, rtol=F32_RTOL, what="diag val")
    parity.assert_rows_close(_np(st), o_st, rtol=F32_RTOL, what="diag state")

    S, Q, Dv, R, k = 600, 120, 48, 16, 80
    src = _t(g.standard_normal((B, S, Dv)), dev, torch.bfloat16)
    qv = _t(g.standard_normal((B, Q, Dv)), dev, torch.bfloat16)
    sstate = _t(g.standard_normal((B, S)), dev, torch.bfloat16)
    w_s = _t(g.standard_normal((R, Dv)) / np.sqrt(Dv), dev, torch.bfloat16)
    w_t = _t(g.standard_normal((R, Dv)) / np.sqrt(Dv), dev, torch.bfloat16)
    core = _t(np.ones(R), dev, torch.bfloat16)
    sender = torch.nn.functional.softplus(sstate.float()).to(torch.bfloat16)
    qs, qvv = jk.transition_query_topk("low_rank_bilinear_route", w_s, None, w_t, None, core, None, None, None,
                                       None, None, 1.0, sender, src, qv, sstate, src, k, 128, 128, True)
    sp = _np((src @ w_s.t()) * core)
    qp = _np(qv @ w_t.t())
    o_st, o_val, _, _ = oracle.transition_query_topk(qp, sp, _np(sstate), _np(src), _np(sender), k)
    parity.assert_rows_close(_np(qvv), o_val, rtol=BF16_RTOL, what="query val")
    parity.assert_rows_close(_np(qs), o_st, rtol=BF16_RTOL, what="query state")

    ts, tv = jk.transition_pairwise_topk("low_rank_bilinear_route", w_s, None, w_t, None, core, None, None, None,
                                         None, None, 1.0, sender, src, qv, sstate, src, k, 128, 128,
                                         route_compress_name="softmax")
    o_ts, o_tv = oracle.transition_pairwise_topk(sp, qp, _np(sstate), _np(src), _np(sender), k)
    parity.assert_rows_close(_np(tv), o_tv, rtol=BF16_RTOL, what="pairwise val")
    parity.assert_rows_close(_np(ts), o_ts, rtol=BF16_RTOL, what="pairwise state")
