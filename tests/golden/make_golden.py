"""Generates the golden fixtures of tests/golden/*.npz by running the reference itself.

    python tests/golden/make_golden.py --reference <path to a Jakal-Net checkout>

Every case builds seeded float32 inputs, runs the reference Layer API with
implementation="reference" (the semantic definition: propagation.py:207-220, 453-480;
transition.py:238-254, 431-452) and stores the inputs, module parameters and outputs.
The window-intersect-top-k case (not a reference operator) is composed from the reference
primitives causal_window_mask / build_topk_mask (kernel_common.py:433-456) and
_compress_edges (propagation.py:67-88). The fixtures pin the CPU oracle
(tests/test_oracle_golden.py); the reference is not needed to run the tests.
"""
from __future__ import annotations

import argparse
from pathlib import Path

import numpy as np
import torch
from torch.nn import functional as F

HERE = Path(__file__).resolve().parent


class TemperatureRoute(torch.nn.Module):
    """Route wrapper exposing `route_fn` / `temperature` like the reference's scaled routes
    (kernel_common.py:117-120 reads exactly these attributes)."""

    expects_pairwise_inputs = True

    def __init__(self, route_fn, temperature):
        super().__init__()
        self.route_fn = route_fn
        self.temperature = temperature

    def forward(self, src, dst):
        return self.route_fn(src, dst) / self.temperature


def _np(t):
    return t.detach().cpu().numpy().astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="Jakal-Net checkout (contains src/jakal_net)")
    args = ap.parse_args()
    import sys

    sys.path.insert(0, str(HERE.parent.parent / "baseline"))
    import reference_shim  # baseline/reference_shim.py

    jn = reference_shim.import_reference(args.reference / "src")
    from jakal_net.kernel_common import build_topk_mask, causal_window_mask
    from jakal_net.kernels import signed_entmax15
    from jakal_net.propagation import _compress_edges

    def signed_abs_softmax(x):
        return torch.sign(torch.nan_to_num(x)) * torch.softmax(torch.nan_to_num(x).abs(), dim=-1)

    signed_abs_softmax.__name__ = "signed_abs_softmax"

    def entmax_edges(x):
        return signed_entmax15(x, dim=-1)

    entmax_edges.__name__ = "signed_entmax15"
    edges = {"softsign": F.softsign, "signed_abs_softmax": signed_abs_softmax, "signed_entmax15": entmax_edges}

    out = {}

    def pairwise(dim, rank, seed):
        torch.manual_seed(seed)
        m = jn.LowRankBilinearPairwise(dim=dim, rank=rank)
        with torch.no_grad():
            m.weight.copy_(torch.rand(rank) + 0.5)
            m.bias.fill_(0.1)
        return m

    def layer(B, N, D, seed):
        g = torch.Generator().manual_seed(seed)
        return jn.Layer(dim=D, num_nodes=N, state=torch.randn(B, N, generator=g), val=torch.randn(B, N, D, generator=g))

    def save_prop(name, m, lay, delta, **extra):
        out[name] = dict(val=_np(lay.val), state=_np(lay.state), w_s=_np(m.source_proj.weight),
                         w_t=_np(m.target_proj.weight), core=_np(m.normalized_weight()), bias=np.float32(m.bias.item()),
                         out_state=_np(delta.delta_state), out_val=_np(delta.delta_val), **extra)

    B, N, D, R = 2, 37, 16, 8
    for ci, (ename, efn) in enumerate(edges.items()):
        m = pairwise(D, R, 10 + ci)
        lay = layer(B, N, D, 20 + ci)
        op = jn.SparsePropagation(pairwise_fn=m, sparse_type="topk", topk=5, edge_compress_fn=efn,
                                  implementation="reference")
        save_prop(f"prop_topk_{ename}", m, lay, op(lay), k=np.int64(5), compress=ename)
        op = jn.SparsePropagation(pairwise_fn=m, sparse_type="window", window=6, edge_compress_fn=efn,
                                  implementation="reference")
        save_prop(f"prop_window_{ename}", m, lay, op(lay), window=np.int64(6), compress=ename)
        op = jn.Propagation(pairwise_fn=m, edge_compress_fn=efn, implementation="reference")
        save_prop(f"prop_dense_{ename}", m, lay, op(lay), compress=ename)

    # state-weighted edges (propagation.py:157-174): edges * softplus(state), state = sum of edges
    m = pairwise(D, R, 30)
    lay = layer(B, N, D, 31)
    op = jn.SparsePropagation(pairwise_fn=m, sparse_type="topk", topk=4, state_weight_edges=True,
                              implementation="reference")
    save_prop("prop_topk_state_weighted", m, lay, op(lay), k=np.int64(4), compress="softsign")

    # window-intersect-top-k from reference primitives
    m = pairwise(D, R, 40)
    lay = layer(B, 45, D, 41)
    with torch.no_grad():
        scores = m(lay.val, lay.val)
        win = causal_window_mask(0, 45, 0, 45, 9).view(1, 45, 45)
        masked = scores.masked_fill(~win, float("-inf"))
        topm = build_topk_mask(masked, 4) & win
        e = _compress_edges(scores, F.softsign, mask=topm)
        d_state = torch.einsum("bij,bj->bi", e, lay.state)
        d_val = torch.einsum("bij,bjd->bid", e, lay.val)
    out["prop_window_topk_softsign"] = dict(val=_np(lay.val), state=_np(lay.state), w_s=_np(m.source_proj.weight),
                                            w_t=_np(m.target_proj.weight), core=_np(m.normalized_weight()),
                                            bias=np.float32(m.bias.item()), out_state=_np(d_state),
                                            out_val=_np(d_val), k=np.int64(4), window=np.int64(9),
                                            compress="softsign")

    # multi-head scorers (modules.py:259-299): per-head low-rank scores combined by max /
    # smoothmax / signed_smoothmax; the raw combined scores and a top-k propagation over them
    for ai, agg in enumerate(("max", "smoothmax", "signed_smoothmax")):
        hs = [pairwise(D, R, 80 + 3 * ai + h) for h in range(3)]
        with torch.no_grad():
            for h, hm in enumerate(hs):
                hm.bias.fill_(0.05 * (h - 1))
        mh = jn.MultiHeadPairwise(hs, aggregate=agg)
        lay = layer(B, N, D, 90 + ai)
        with torch.no_grad():
            scores = mh(lay.val, lay.val)
        op = jn.SparsePropagation(pairwise_fn=mh, sparse_type="topk", topk=5, implementation="reference")
        delta = op(lay)
        out[f"multihead_{agg}"] = dict(
            val=_np(lay.val), state=_np(lay.state), w_s=np.stack([_np(h.source_proj.weight) for h in hs]),
            w_t=np.stack([_np(h.target_proj.weight) for h in hs]), core=np.stack([_np(h.normalized_weight()) for h in hs]),
            bias=np.array([h.bias.item() for h in hs], np.float32), scores=_np(scores), k=np.int64(5),
            compress="softsign", out_state=_np(delta.delta_state), out_val=_np(delta.delta_val))

    # diagonal bilinear scorer / route (modules.py:37-53, 385-412)
    torch.manual_seed(95)
    dm = jn.DiagonalBilinearPairwise(D)
    with torch.no_grad():
        dm.weight.copy_(torch.rand(D) + 0.5)
        dm.bias.fill_(0.07)
    lay = layer(B, N, D, 96)
    op = jn.SparsePropagation(pairwise_fn=dm, sparse_type="topk", topk=5, implementation="reference")
    delta = op(lay)
    out["prop_topk_diagonal"] = dict(val=_np(lay.val), state=_np(lay.state), core=_np(dm.normalized_weight()),
                                     bias=np.float32(dm.bias.item()), k=np.int64(5), compress="softsign",
                                     out_state=_np(delta.delta_state), out_val=_np(delta.delta_val))
    torch.manual_seed(97)
    dr = jn.DiagonalBilinearRoute(D, D)
    with torch.no_grad():
        dr.weight.copy_(torch.rand(D) + 0.5)
        dr.bias.fill_(-0.1)
    src = layer(B, 29, D, 98)
    dst = layer(B, 11, D, 99)
    op = jn.SparseTransition(route_fn=dr, topk=3, route_compress_name="softmax", implementation="reference")
    delta = op.compute_delta(src, dst)
    out["transition_topk_diagonal"] = dict(
        src_val=_np(src.val), src_state=_np(src.state), dst_val=_np(dst.val), core=_np(dr.normalized_weight()),
        bias=np.float32(dr.bias.item()), temperature=np.float32(1.0), k=np.int64(3), compress="softmax",
        out_state=_np(delta.delta_state), out_val=_np(delta.delta_val))

    # transitions with a low-rank route
    def route(src_dim, dst_dim, rank, seed, temperature):
        torch.manual_seed(seed)
        r = jn.LowRankBilinearRoute(src_dim, dst_dim, rank=rank)
        with torch.no_grad():
            r.weight.copy_(torch.rand(rank) + 0.5)
            r.bias.fill_(-0.2)
        return r, (TemperatureRoute(r, temperature) if temperature != 1.0 else r)

    S, Q = 29, 11
    for ci, (rname, temp) in enumerate((("softmax", 1.0), ("signed_abs_softmax", 0.7), ("signed_entmax15", 1.0))):
        r, rf = route(D, D, R, 50 + ci, temp)
        src = layer(B, S, D, 60 + ci)
        dst = layer(B, Q, D, 70 + ci)
        op = jn.SparseTransition(route_fn=rf, topk=3, route_compress_name=rname, implementation="reference")
        delta = op.compute_delta(src, dst)
        out[f"transition_topk_{rname}"] = dict(
            src_val=_np(src.val), src_state=_np(src.state), dst_val=_np(dst.val), w_s=_np(r.source_proj.weight),
            w_t=_np(r.target_proj.weight), core=_np(r.weight), bias=np.float32(r.bias.item()),
            temperature=np.float32(temp), k=np.int64(3), compress=rname,
            out_state=_np(delta.delta_state), out_val=_np(delta.delta_val))
        op = jn.Transition(route_fn=rf, route_compress_name=rname, implementation="reference")
        delta = op.compute_delta(src, dst)
        out[f"transition_dense_{rname}"] = dict(
            src_val=_np(src.val), src_state=_np(src.state), dst_val=_np(dst.val), w_s=_np(r.source_proj.weight),
            w_t=_np(r.target_proj.weight), core=_np(r.weight), bias=np.float32(r.bias.item()),
            temperature=np.float32(temp), compress=rname,
            out_state=_np(delta.delta_state), out_val=_np(delta.delta_val))

    for name, arrays in out.items():
        np.savez(HERE / f"{name}.npz", **{k: np.asarray(v) for k, v in arrays.items()})
        print("wrote", name)


if __name__ == "__main__":
    main()
