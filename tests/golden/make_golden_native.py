"""Generates tests/golden/query_topk_*.npz by running the reference's own native extension.

    python oracle/build_ref.py --cpu && python tests/golden/make_golden_native.py

The per-query transition (transition_query_topk, jakal_net_native.cpp:7089-7246) has no
Python Layer-API class in the reference, so its only executable definition is the native
op itself. This script calls the CPU build of it (oracle/_ref/cpu, built from the
reference's sources by oracle/build_ref.py) on seeded f32 inputs through the positional
signature native_backend.py:5919-5941 uses, and stores inputs and outputs. The fixtures pin
the oracle's transition_query_topk (tests/test_oracle_golden.py); the reference and its
build are not needed to run the tests.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
import build_ref  # noqa: E402  (oracle/build_ref.py)


def _np(t):
    return t.detach().cpu().numpy().astype(np.float32)


def main():
    native = build_ref.load_built("cpu")
    assert native.backend_name() == "aten_cpp_cpu"
    out = {}
    B, S, Q, D, R = 2, 53, 13, 16, 8
    for name, kind, temperature, k, qblock, sblock in (
        ("query_topk_low_rank", "low_rank_bilinear_route", 0.7, 5, 4, 16),
        ("query_topk_low_rank_k_all", "low_rank_bilinear_route", 1.0, 60, 0, 0),
        ("query_topk_diagonal", "diagonal_bilinear_route", 1.0, 7, 5, 11),
    ):
        g = torch.Generator().manual_seed(len(out) + 300)
        src = torch.randn(B, S, D, generator=g)
        qv = 0.5 * torch.randn(B, Q, D, generator=g)
        pstate = torch.randn(B, S, generator=g)
        pval = torch.randn(B, S, D, generator=g)
        sender = torch.nn.functional.softplus(torch.randn(B, S, generator=g))
        core = torch.rand(R if kind.startswith("low") else D, generator=g) + 0.5
        bias = torch.tensor(-0.15)
        if kind == "low_rank_bilinear_route":
            w_s = torch.randn(R, D, generator=g) / D ** 0.5
            w_t = torch.randn(R, D, generator=g) / D ** 0.5
        else:
            w_s = w_t = None
        st, vv = native.transition_query_topk(kind, w_s, None, w_t, None, core, bias, None, None, None, None,
                                                      float(temperature), sender, src, qv, pstate, pval, k, qblock,
                                                      sblock, False)
        case = dict(src_val=_np(src), query_val=_np(qv), state=_np(pstate), val=_np(pval), sender=_np(sender),
                    core=_np(core), bias=np.float32(bias.item()), temperature=np.float32(temperature),
                    k=np.int64(k), kind=kind, out_state=_np(st), out_val=_np(vv))
        if w_s is not None:
            case.update(w_s=_np(w_s), w_t=_np(w_t))
        out[name] = case
    for name, arrays in out.items():
        np.savez(HERE / f"{name}.npz", **{k: np.asarray(v) for k, v in arrays.items()})
        print("wrote", name)


if __name__ == "__main__":
    main()
