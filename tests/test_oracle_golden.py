"""Pins the CPU oracle: against fixtures produced by the reference implementation itself
(tests/golden/make_golden.py) and against the reference's own known-answer tests."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
RTOL, ATOL = 1e-4, 2e-5


def _load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    return {k: z[k] for k in z.files}


def _prop_projections(g):
    pt = oracle.lowrank_project(g["val"], g["w_t"], None, 1.0, "f32")
    ps = oracle.lowrank_project(g["val"], g["w_s"], g["core"], 1.0, "f32")
    return pt, ps


def _close(got, ref):
    np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("compress", ["softsign", "signed_abs_softmax", "signed_entmax15"])
def test_propagation_topk_matches_reference(compress):
    g = _load(f"prop_topk_{compress}")
    pt, ps = _prop_projections(g)
    st, val, _, _ = oracle.propagation_topk(pt, ps, g["state"], g["val"], int(g["k"]), bias=float(g["bias"]),
                                            compress_name=compress)
    _close(st, g["out_state"])
    _close(val, g["out_val"])


@pytest.mark.parametrize("compress", ["softsign", "signed_abs_softmax", "signed_entmax15"])
def test_propagation_window_matches_reference(compress):
    g = _load(f"prop_window_{compress}")
    pt, ps = _prop_projections(g)
    st, val = oracle.propagation_masked_dense(pt, ps, g["state"], g["val"], window=int(g["window"]),
                                              bias=float(g["bias"]), compress_name=compress)
    _close(st, g["out_state"])
    _close(val, g["out_val"])


@pytest.mark.parametrize("compress", ["softsign", "signed_abs_softmax", "signed_entmax15"])
def test_propagation_dense_matches_reference(compress):
    g = _load(f"prop_dense_{compress}")
    pt, ps = _prop_projections(g)
    st, val = oracle.propagation_masked_dense(pt, ps, g["state"], g["val"], window=None, bias=float(g["bias"]),
                                              compress_name=compress)
    _close(st, g["out_state"])
    _close(val, g["out_val"])


def test_state_weighted_topk_matches_reference():
    # propagation.py:165-174: projected_state = softplus(state), projected_val = val * softplus(state)
    g = _load("prop_topk_state_weighted")
    pt, ps = _prop_projections(g)
    strength = oracle.softplus(g["state"])
    st, val, _, _ = oracle.propagation_topk(pt, ps, strength, g["val"] * strength[..., None], int(g["k"]),
                                            bias=float(g["bias"]))
    _close(st, g["out_state"])
    _close(val, g["out_val"])


def test_window_intersect_topk_matches_reference_primitives():
    g = _load("prop_window_topk_softsign")
    pt, ps = _prop_projections(g)
    st, val, _, _ = oracle.propagation_topk(pt, ps, g["state"], g["val"], int(g["k"]), window=int(g["window"]),
                                            bias=float(g["bias"]))
    _close(st, g["out_state"])
    _close(val, g["out_val"])


def _route(g):
    T = float(g["temperature"])
    src = oracle.lowrank_project(g["src_val"], g["w_s"], g["core"], T, "f32")
    dst = oracle.lowrank_project(g["dst_val"], g["w_t"], None, 1.0, "f32")
    return src, dst, float(g["bias"]) / T


@pytest.mark.parametrize("compress", ["softmax", "signed_abs_softmax", "signed_entmax15"])
def test_sparse_transition_matches_reference(compress):
    g = _load(f"transition_topk_{compress}")
    src, dst, bias = _route(g)
    st, val = oracle.transition_pairwise_topk(src, dst, g["src_state"], g["src_val"], oracle.softplus(g["src_state"]),
                                              int(g["k"]), bias=bias, compress_name=compress)
    _close(st, g["out_state"])
    _close(val, g["out_val"])


@pytest.mark.parametrize("compress", ["softmax", "signed_abs_softmax", "signed_entmax15"])
def test_dense_transition_matches_reference(compress):
    g = _load(f"transition_dense_{compress}")
    src, dst, bias = _route(g)
    st, val = oracle.transition_dense(src, dst, g["src_state"], g["src_val"], oracle.softplus(g["src_state"]),
                                      bias=bias, compress_name=compress)
    _close(st, g["out_state"])
    _close(val, g["out_val"])


# ---- known-answer tests of the reference (tests/test_jakal_net.py)
def test_kat_propagation_has_no_state_activation():
    # tests/test_jakal_net.py:438-458: all-ones scores, softsign -> edges 0.5
    scores = np.ones((1, 2, 2))
    st, val = oracle.masked_dense_from_scores(scores, np.array([[-1.0, 2.0]]), np.array([[[1.0], [3.0]]]),
                                              window=None)
    np.testing.assert_allclose(st, [[0.5, 0.5]])
    np.testing.assert_allclose(val, [[[2.0], [2.0]]])


def test_kat_transition_routes_with_state_activation():
    # tests/test_jakal_net.py:810-831: zero logits, softmax, sender = state + 1, added to dst
    state = np.array([[1.0, 2.0]])
    val = np.array([[[1.0, 0.0], [0.0, 2.0]]])
    st, v = oracle.dense_transition_from_logits(np.zeros((1, 2, 2)), state, val, state + 1.0)
    np.testing.assert_allclose(st, [[4.0, 4.0]])
    np.testing.assert_allclose(v, [[[1.0, 3.0], [1.0, 3.0]]])


def test_kat_sparse_transition_uses_topk_before_softmax():
    # tests/test_jakal_net.py:833-862: topk=1 picks one destination per source, route 1
    logits = np.array([[[3.0, 1.0, 0.0], [0.0, 2.0, 4.0]]])
    state = np.array([[1.0, 2.0]])
    val = np.array([[[10.0], [20.0]]])
    st, v = oracle.sparse_transition_from_logits(logits, state, val, state + 1.0, 1)
    dst_state = np.array([[5.0, 5.0, 5.0]]) + st
    dst_val = np.ones((1, 3, 1)) + v
    np.testing.assert_allclose(dst_state, [[7.0, 5.0, 11.0]])
    np.testing.assert_allclose(dst_val, [[[21.0], [1.0], [61.0]]])


def test_topk_tie_order_prefers_lower_index():
    scores = np.zeros((1, 1, 6))
    _, _, _, idx = oracle.topk_from_scores(scores, np.zeros((1, 6)), np.zeros((1, 6, 1)), 3)
    assert idx.tolist() == [[[0, 1, 2]]]


def test_round_bf16_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, 1.0 + 2 ** -9, -3.14159], np.float32)
    r = oracle.round_to(x, "bf16")
    import torch

    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(r, ref)


def test_entmax15_sums_to_one_and_is_sparse():
    p = oracle.entmax15(np.array([3.0, 1.0, 0.2, -1.0]))
    assert abs(p.sum() - 1.0) < 1e-12
    assert p[-1] == 0.0


def _multihead_projections(g, dtype="f32"):
    """Per-head projections [B, H, N, R] of a multi-head fixture."""
    H = g["w_s"].shape[0]
    pt = np.stack([oracle.lowrank_project(g["val"], g["w_t"][h], None, 1.0, dtype) for h in range(H)], axis=1)
    ps = np.stack([oracle.lowrank_project(g["val"], g["w_s"][h], g["core"][h], 1.0, dtype) for h in range(H)], axis=1)
    return pt, ps


@pytest.mark.parametrize("combine", ["max", "smoothmax", "signed_smoothmax"])
def test_multihead_scores_match_reference(combine):
    g = _load(f"multihead_{combine}")
    pt, ps = _multihead_projections(g)
    _close(oracle.multihead_scores(pt, ps, g["bias"], combine), g["scores"])


@pytest.mark.parametrize("combine", ["max", "smoothmax", "signed_smoothmax"])
def test_multihead_topk_propagation_matches_reference(combine):
    g = _load(f"multihead_{combine}")
    pt, ps = _multihead_projections(g)
    scores = oracle.multihead_scores(pt, ps, g["bias"], combine)
    st, val, _, _ = oracle.topk_from_scores(scores, g["state"], g["val"], int(g["k"]), compress_name="softsign")
    _close(st, g["out_state"])
    _close(val, g["out_val"])


def test_diagonal_topk_propagation_matches_reference():
    g = _load("prop_topk_diagonal")
    scores = oracle.lowrank_scores(g["val"], g["val"] * g["core"], float(g["bias"]))
    st, val, _, _ = oracle.topk_from_scores(scores, g["state"], g["val"], int(g["k"]), compress_name="softsign")
    _close(st, g["out_state"])
    _close(val, g["out_val"])


def test_diagonal_route_transition_matches_reference():
    g = _load("transition_topk_diagonal")
    logits = oracle.lowrank_scores(g["src_val"] * g["core"], g["dst_val"], float(g["bias"]))
    st, val = oracle.sparse_transition_from_logits(logits, g["src_state"], g["src_val"], oracle.softplus(g["src_state"]),
                                                   int(g["k"]), compress_name="softmax")
    _close(st, g["out_state"])
    _close(val, g["out_val"])


@pytest.mark.parametrize("name", ["query_topk_low_rank", "query_topk_low_rank_k_all", "query_topk_diagonal"])
def test_transition_query_topk_matches_reference_native_build(name):
    """Per-query transition pinned to the reference's own native op (CPU build of
    jakal_net_native.cpp:7089-7246; fixtures from tests/golden/make_golden_native.py):
    logits route(src, query)^T / T + b / T, top-k sources per query, softmax over the k,
    sender-weighted gather."""
    g = _load(name)
    T = float(g["temperature"])
    if str(g["kind"]) == "low_rank_bilinear_route":
        sp = oracle.lowrank_project(g["src_val"], g["w_s"], g["core"], T, "f32")
        qp = oracle.lowrank_project(g["query_val"], g["w_t"], None, 1.0, "f32")
    else:
        sp = oracle.lowrank_project(g["src_val"], np.eye(g["src_val"].shape[-1]), g["core"], T, "f32")
        qp = g["query_val"].astype(np.float64)
    k = min(int(g["k"]), g["src_val"].shape[1])
    st, val, _, _ = oracle.transition_query_topk(qp, sp, g["state"], g["val"], g["sender"], k,
                                                 bias=float(g["bias"]) / T)
    _close(st, g["out_state"])
    _close(val, g["out_val"])
