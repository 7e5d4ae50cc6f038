"""GPU ops against the reference's own outputs (tests/golden, produced by running the
reference implementation on f32 inputs): the f32 path of the module, end to end through
the C ABI, with the reference's test tolerance scale (1e-4 of the row magnitude)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import parity

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
RTOL = 1e-4


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda", 0)


def _load(name, dev):
    z = np.load(GOLDEN / f"{name}.npz")
    out = {}
    for k in z.files:
        a = z[k]
        out[k] = torch.from_numpy(a).to(dev) if a.dtype.kind == "f" and a.ndim > 0 else a
    return out


def _check(st, vv, g):
    parity.assert_rows_close(vv.float().cpu().numpy(), g["out_val"].cpu().numpy(), rtol=RTOL, what="val")
    parity.assert_rows_close(st.float().cpu().numpy(), g["out_state"].cpu().numpy(), rtol=RTOL, what="state")


def _spec(g, dev):
    return ("low_rank_bilinear", g["core"], torch.tensor(float(g["bias"]), device=dev), g["w_s"], None, g["w_t"], None)


@pytest.mark.parametrize("compress", ["softsign", "signed_abs_softmax", "signed_entmax15"])
def test_topk_matches_reference(dev, compress):
    import jakal_net_b200 as jk

    g = _load(f"prop_topk_{compress}", dev)
    st, vv = jk.propagation_topk(*_spec(g, dev), compress, g["val"], g["state"], g["val"], int(g["k"]), 128, 128)
    _check(st, vv, g)


@pytest.mark.parametrize("compress", ["softsign", "signed_abs_softmax", "signed_entmax15"])
def test_window_matches_reference(dev, compress):
    import jakal_net_b200 as jk

    g = _load(f"prop_window_{compress}", dev)
    st, vv = jk.propagation_window(*_spec(g, dev), compress, g["val"], g["state"], g["val"], int(g["window"]), 128,
                                   128)
    _check(st, vv, g)


@pytest.mark.parametrize("compress", ["softsign", "signed_abs_softmax", "signed_entmax15"])
def test_dense_matches_reference(dev, compress):
    import jakal_net_b200 as jk

    g = _load(f"prop_dense_{compress}", dev)
    st, vv = jk.propagation_dense(*_spec(g, dev), compress, g["val"], g["state"], g["val"], None, 128, 128)
    _check(st, vv, g)


def test_state_weighted_topk_matches_reference(dev):
    import jakal_net_b200 as jk

    g = _load("prop_topk_state_weighted", dev)
    strength = torch.nn.functional.softplus(g["state"])
    st, vv = jk.propagation_topk(*_spec(g, dev), "softsign", g["val"], strength, g["val"] * strength[..., None],
                                 int(g["k"]), 128, 128)
    _check(st, vv, g)


def test_window_intersect_topk_matches_reference_primitives(dev):
    import jakal_net_b200 as jk

    g = _load("prop_window_topk_softsign", dev)
    st, vv = jk.propagation_window_topk(*_spec(g, dev), "softsign", g["val"], g["state"], g["val"],
                                        int(g["window"]), int(g["k"]))
    _check(st, vv, g)


@pytest.mark.parametrize("compress", ["softmax", "signed_abs_softmax", "signed_entmax15"])
def test_sparse_transition_matches_reference(dev, compress):
    import jakal_net_b200 as jk

    g = _load(f"transition_topk_{compress}", dev)
    sender = torch.nn.functional.softplus(g["src_state"])
    st, vv = jk.transition_pairwise_topk("low_rank_bilinear_route", g["w_s"], None, g["w_t"], None, g["core"],
                                         torch.tensor(float(g["bias"]), device=dev), None, None, None, None,
                                         float(g["temperature"]), sender, g["src_val"], g["dst_val"], g["src_state"],
                                         g["src_val"], int(g["k"]), 128, 128, route_compress_name=compress)
    _check(st, vv, g)


@pytest.mark.parametrize("compress", ["softmax", "signed_abs_softmax", "signed_entmax15"])
def test_dense_transition_matches_reference(dev, compress):
    import jakal_net_b200 as jk

    g = _load(f"transition_dense_{compress}", dev)
    sender = torch.nn.functional.softplus(g["src_state"])
    st, vv = jk.transition_pairwise_dense("low_rank_bilinear_route", g["w_s"], None, g["w_t"], None, g["core"],
                                          torch.tensor(float(g["bias"]), device=dev), None, None, None, None,
                                          compress, float(g["temperature"]), sender, g["src_val"], g["dst_val"],
                                          g["src_state"], g["src_val"], 128, 128)
    _check(st, vv, g)


def test_diagonal_topk_matches_reference(dev):
    import jakal_net_b200 as jk

    g = _load("prop_topk_diagonal", dev)
    st, vv = jk.propagation_topk("diagonal_bilinear", g["core"], torch.tensor(float(g["bias"]), device=dev), None,
                                 None, None, None, "softsign", g["val"], g["state"], g["val"], int(g["k"]), 128, 128)
    _check(st, vv, g)


def test_diagonal_route_transition_matches_reference(dev):
    import jakal_net_b200 as jk

    g = _load("transition_topk_diagonal", dev)
    sender = torch.nn.functional.softplus(g["src_state"])
    st, vv = jk.transition_pairwise_topk("diagonal_bilinear_route", None, None, None, None, g["core"],
                                         torch.tensor(float(g["bias"]), device=dev), None, None, None, None,
                                         float(g["temperature"]), sender, g["src_val"], g["dst_val"], g["src_state"],
                                         g["src_val"], int(g["k"]), 128, 128, route_compress_name="softmax")
    _check(st, vv, g)
