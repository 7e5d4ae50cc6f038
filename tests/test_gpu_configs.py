"""GPU parity at the benchmark configurations' own shapes (bf16, seeded), against the oracle.

* config 2: B8 N2048 D384 R64, causal window 512 intersect top-k 32 -- the bench workload,
  every row checked (selection and outputs);
* config 3: per-query transition B16, S 4096 x 512 sources, Q 512 slots, R64, k16 -- the
  public op, every query slot checked;
* config 5: one batch item of N32768 D512 R64, window 4096, k64 -- the public op on the full
  sequence, checked on a sample of rows that covers every kind of tile boundary (first rows,
  the 128-row CTA edges, the window edge at 4096, the last rows) plus random rows.
The oracle runs on the library's own bf16 projections, so the fused kernel is isolated (the
projection kernel has its own test); outputs are bf16, hence one bf16 rounding step on top of
the kernel tolerance."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import parity

pytestmark = pytest.mark.gpu
OUT_RTOL = parity.VAL_RTOL + 2 ** -8


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda", 0)


def _gen(seed, dev):
    g = torch.Generator().manual_seed(seed)

    def randn(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(dev, torch.bfloat16)

    return randn


def _np(t):
    return t.detach().double().cpu().numpy()


def test_config2_full_batch(dev):
    import jakal_net_b200 as jk

    B, N, D, R, W, k = 8, 2048, 384, 64, 512, 32
    randn = _gen(1, dev)
    val, state = randn(B, N, D), randn(B, N)
    w_s, w_t = randn(R, D, scale=D ** -0.5), randn(R, D, scale=D ** -0.5)
    core = torch.full((R,), R ** -0.5, device=dev)
    st, vv = jk.propagation_window_topk("low_rank_bilinear", core, None, w_s, None, w_t, None, "softsign", val,
                                        state, val, W, k)
    pt = jk.lowrank_project(val, w_t)
    ps = jk.lowrank_project(val, w_s, core=core)
    _, _, sc, ix = jk.topk_aggregate(pt, ps, state, val, k, window=W, return_selection=True)
    torch.cuda.synchronize()
    rp, cp = _np(pt), _np(ps)
    o_st, o_val, o_sc, o_ix = oracle.propagation_topk(rp, cp, _np(state), _np(val), k, window=W)
    parity.set_full_scores(oracle.lowrank_scores(rp, cp, 0.0))
    ties = parity.tie_rows(ix.cpu().numpy(), o_ix, o_sc)
    assert ties.mean() < 0.01
    parity.assert_rows_close(_np(vv), o_val, ties, rtol=OUT_RTOL, what="config 2 val")
    parity.assert_rows_close(_np(st), o_st, ties, rtol=OUT_RTOL, what="config 2 state")


def test_config3_query_transition(dev):
    import jakal_net_b200 as jk

    B, S, Q, D, R, k = 16, 4096, 512, 512, 64, 16
    randn = _gen(2, dev)
    src, sstate = randn(B, S, D), randn(B, S)
    qv = randn(B, Q, D, scale=0.02)
    w_s, w_t = randn(R, D, scale=D ** -0.5), randn(R, D, scale=D ** -0.5)
    core = torch.ones(R, device=dev, dtype=torch.bfloat16)
    sender = torch.nn.functional.softplus(sstate.float()).to(torch.bfloat16)
    st, vv = jk.transition_query_topk("low_rank_bilinear_route", w_s, None, w_t, None, core, None, None, None, None,
                                      None, 1.0, sender, src, qv, sstate, src, k, 128, 128, True)
    torch.cuda.synchronize()
    sp = _np(jk.lowrank_project(src, w_s, core=core))
    qp = _np(jk.lowrank_project(qv, w_t))
    o_st, o_val, _, _ = oracle.transition_query_topk(qp, sp, _np(sstate), _np(src), _np(sender), k)
    parity.assert_rows_close(_np(vv), o_val, rtol=OUT_RTOL, what="config 3 val")
    parity.assert_rows_close(_np(st), o_st, rtol=OUT_RTOL, what="config 3 state")


def test_config5_sampled_rows(dev):
    import jakal_net_b200 as jk

    N, D, R, W, k = 32768, 512, 64, 4096, 64
    randn = _gen(4, dev)
    val, state = randn(1, N, D), randn(1, N)
    w_s, w_t = randn(R, D, scale=D ** -0.5), randn(R, D, scale=D ** -0.5)
    core = torch.full((R,), R ** -0.5, device=dev)
    st, vv = jk.propagation_window_topk("low_rank_bilinear", core, None, w_s, None, w_t, None, "softsign", val,
                                        state, val, W, k)
    torch.cuda.synchronize()
    rp = _np(jk.lowrank_project(val, w_t))[0]
    cp = _np(jk.lowrank_project(val, w_s, core=core))[0]
    sv, vals = _np(state)[0], _np(val)[0]
    edges = [0, 1, 2, 63, 64, 127, 128, 129, 255, 256, 4095, 4096, 4097, 4223, 4224, 16383, 16384, N - 129,
             N - 128, N - 2, N - 1]
    rows = sorted(set(edges) | set(np.random.default_rng(5).integers(0, N, 200).tolist()))
    got_st, got_val = _np(st)[0], _np(vv)[0]
    want_st = np.zeros(len(rows))
    want_val = np.zeros((len(rows), D))
    for i, t in enumerate(rows):
        lo = max(0, t - W)
        sc = cp[lo:t + 1] @ rp[t]
        vis = np.ones(sc.shape[0], dtype=bool)
        idx = oracle.select_topk(sc, vis, k)
        e = oracle.compress(sc[idx], "softsign")
        want_st[i] = e @ sv[lo + idx]
        want_val[i] = e @ vals[lo + idx]
    parity.assert_rows_close(got_val[rows], want_val, rtol=OUT_RTOL, what="config 5 val")
    parity.assert_rows_close(got_st[rows][None], want_st[None], rtol=OUT_RTOL, what="config 5 state")
