"""GPU parity of the multi-head scorers (MultiHeadPairwise / MultiHeadRoute, modules.py:259-302;
spec kinds multihead_{max,smoothmax,signed_smoothmax}_low_rank_bilinear and
multihead_max_low_rank_bilinear_route, kernel_common.py:151-178, 238-273) against the CPU
oracle, through the C ABI (*_mh entry points), on seeded bf16 inputs.

The oracle scores come from the per-head blocks of the same packed bf16 projections the
library used (jakal_net_b200._multihead_project); oracle.multihead_scores is pinned to the
reference's own MultiHeadPairwise outputs by tests/test_oracle_golden.py."""
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


def _heads(g, H, R, D, dev):
    w_s = _t(g.standard_normal((H, R, D)) / np.sqrt(D), dev)
    w_t = _t(g.standard_normal((H, R, D)) / np.sqrt(D), dev)
    core = _t(np.abs(g.standard_normal((H, R))) / np.sqrt(R) + 0.05, dev)
    bias = torch.tensor(np.linspace(-0.1, 0.1, H), device=dev, dtype=torch.float32)
    return w_s, w_t, core, bias


def _unpack(proj, H, R):
    """[B, N, rp] packed head blocks -> [B, H, N, R] (head h at columns 16 kph h .. + R)."""
    p = _np(proj)
    rb = -(-R // 16) * 16
    return np.stack([p[..., h * rb:h * rb + R] for h in range(H)], axis=1)


def _scores(jk, t_val, s_val, w_t, w_s, core, bias, combine, temperature=1.0):
    rp_t, _ = jk._multihead_project(t_val, w_t)
    rp_s, _ = jk._multihead_project(s_val, w_s, core=core, temperature=temperature)
    H, R = core.shape
    return oracle.multihead_scores(_unpack(rp_t, H, R), _unpack(rp_s, H, R), _np(bias) / temperature, combine)


def _close(st, vv, o_st, o_val):
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="state")


@pytest.mark.parametrize("combine", ["max", "smoothmax", "signed_smoothmax"])
@pytest.mark.parametrize("H,R", [(2, 32), (4, 32), (3, 16)])
def test_multihead_topk_propagation(dev, combine, H, R):
    import jakal_net_b200 as jk

    g = np.random.default_rng(100 + H * R)
    B, N, D, k = 2, 520, 128, 16
    val = _t(g.standard_normal((B, N, D)), dev)
    state = _t(g.standard_normal((B, N)), dev)
    w_s, w_t, core, bias = _heads(g, H, R, D, dev)
    kind = f"multihead_{combine}_low_rank_bilinear"
    st, vv = jk.propagation_topk(kind, core, bias, w_s, None, w_t, None, "softsign", val, state, val, k, 128, 128)
    sc = _scores(jk, val, val, w_t, w_s, core, bias, combine)
    o_st, o_val, _, _ = oracle.topk_from_scores(sc, _np(state), _np(val), k, compress_name="softsign")
    _close(st, vv, o_st, o_val)


@pytest.mark.parametrize("combine", ["max", "signed_smoothmax"])
def test_multihead_window_topk_propagation(dev, combine):
    import jakal_net_b200 as jk

    g = np.random.default_rng(7)
    B, N, D, H, R, W, k = 2, 700, 192, 2, 64, 300, 32
    val = _t(g.standard_normal((B, N, D)), dev)
    state = _t(g.standard_normal((B, N)), dev)
    w_s, w_t, core, bias = _heads(g, H, R, D, dev)
    kind = f"multihead_{combine}_low_rank_bilinear"
    st, vv = jk.propagation_window_topk(kind, core, bias, w_s, None, w_t, None, "signed_abs_softmax", val, state, val,
                                        W, k)
    sc = _scores(jk, val, val, w_t, w_s, core, bias, combine)
    o_st, o_val, _, _ = oracle.topk_from_scores(sc, _np(state), _np(val), k, window=W,
                                                compress_name="signed_abs_softmax")
    _close(st, vv, o_st, o_val)


@pytest.mark.parametrize("combine", ["max", "smoothmax", "signed_smoothmax"])
@pytest.mark.parametrize("W", [90, -1])
def test_multihead_window_and_dense_propagation(dev, combine, W):
    import jakal_net_b200 as jk

    g = np.random.default_rng(300 + W)
    B, N, D, H, R = 2, 333, 128, 2, 32
    val = _t(g.standard_normal((B, N, D)), dev)
    state = _t(g.standard_normal((B, N)), dev)
    w_s, w_t, core, bias = _heads(g, H, R, D, dev)
    kind = f"multihead_{combine}_low_rank_bilinear"
    if W >= 0:
        st, vv = jk.propagation_window(kind, core, bias, w_s, None, w_t, None, "signed_entmax15", val, state, val, W,
                                       128, 128)
    else:
        st, vv = jk.propagation_dense(kind, core, bias, w_s, None, w_t, None, "signed_entmax15", val, state, val,
                                      None, 128, 128)
    sc = _scores(jk, val, val, w_t, w_s, core, bias, combine)
    o_st, o_val = oracle.masked_dense_from_scores(sc, _np(state), _np(val), window=None if W < 0 else W,
                                                  compress_name="signed_entmax15")
    _close(st, vv, o_st, o_val)


def test_multihead_route_transitions(dev):
    import jakal_net_b200 as jk

    g = np.random.default_rng(55)
    B, S, Q, D, H, R, k, T = 2, 600, 150, 128, 2, 32, 8, 0.7
    src = _t(g.standard_normal((B, S, D)), dev)
    dst = _t(g.standard_normal((B, Q, D)), dev)
    sstate = _t(g.standard_normal((B, S)), dev)
    w_s, w_t, core, bias = _heads(g, H, R, D, dev)
    sender = torch.nn.functional.softplus(sstate.float()).to(torch.bfloat16)
    kind = "multihead_max_low_rank_bilinear_route"
    # route logits [B, S, Q] = (ps_h . pd_h + b_h) / T, max over heads (sources carry core and 1/T)
    ps, _ = jk._multihead_project(src, w_s, core=core, temperature=T)
    pd, _ = jk._multihead_project(dst, w_t)
    logits = oracle.multihead_scores(_unpack(ps, H, R), _unpack(pd, H, R), _np(bias) / T, "max")
    # per-query top-k: queries pick sources
    st, vv = jk.transition_query_topk(kind, w_s, None, w_t, None, core, bias, None, None, None, None, T, sender, src,
                                      dst, sstate, src, k, 128, 128, True)
    o_st, o_val, _, _ = oracle.topk_from_scores(np.swapaxes(logits, 1, 2), _np(sstate), _np(src), k,
                                                compress_name="softmax", col_sender=_np(sender))
    _close(st, vv, o_st, o_val)
    # per-source top-k scatter
    st, vv = jk.transition_pairwise_topk(kind, w_s, None, w_t, None, core, bias, None, None, None, None, T, sender,
                                         src, dst, sstate, src, k, 128, 128, route_compress_name="softmax")
    o_st, o_val = oracle.sparse_transition_from_logits(logits, _np(sstate), _np(src), _np(sender), k,
                                                       compress_name="softmax")
    _close(st, vv, o_st, o_val)
    # dense
    st, vv = jk.transition_pairwise_dense(kind, w_s, None, w_t, None, core, bias, None, None, None, None, "softmax", T,
                                          sender, src, dst, sstate, src, 128, 128)
    o_st, o_val = oracle.dense_transition_from_logits(logits, _np(sstate), _np(src), _np(sender),
                                                      compress_name="softmax")
    _close(st, vv, o_st, o_val)
