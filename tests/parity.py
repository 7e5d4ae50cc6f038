"""Parity helpers shared by the GPU tests: tolerance rules written once.

Rules:
* top-k index sets must be identical, except where the oracle's scores of the differing
  columns are within 1e-5 relative of the row's k-th best score (a tie);
* values and states within 2e-3 relative per element (against the element's magnitude plus
  its row's rms, the floor for near-zero sums) for bf16 / f16 inputs with f32
  accumulation, on rows without a tie.
"""
from __future__ import annotations

import numpy as np

TIE_RTOL = 1e-5
VAL_RTOL = 2e-3


def tie_rows(gpu_index: np.ndarray, ora_index: np.ndarray, ora_scores: np.ndarray) -> np.ndarray:
    """Boolean [B, T]: rows whose index sets differ. Raises if a difference is not a tie."""
    B, T, k = gpu_index.shape
    diff = np.zeros((B, T), dtype=bool)
    for b in range(B):
        for t in range(T):
            g = set(int(i) for i in gpu_index[b, t] if i >= 0)
            o = set(int(i) for i in ora_index[b, t] if i >= 0)
            if g == o:
                continue
            diff[b, t] = True
            n = len(o)
            assert len(g) == n, f"row {(b, t)}: selected {len(g)} vs oracle {n}"
            kth = ora_scores[b, t, n - 1]
            tol = TIE_RTOL * max(1.0, abs(kth))
            for j in g ^ o:
                # score of column j as the oracle computes it
                sj = ora_scores_lookup(b, t, j)
                assert abs(sj - kth) <= tol, f"row {(b, t)} column {j}: score {sj} vs k-th {kth} is not a tie"
    return diff


_LOOKUP = {}


def ora_scores_lookup(b, t, j):
    return _LOOKUP["scores"][b, t, j]


def set_full_scores(scores: np.ndarray) -> None:
    _LOOKUP["scores"] = scores


def assert_rows_close(gpu: np.ndarray, ref: np.ndarray, skip_rows: np.ndarray | None = None, rtol: float = VAL_RTOL,
                      what: str = "") -> None:
    """Per-element relative check: |gpu - ref| <= rtol * (|ref| + rms(ref row)).

    The row of an element is its value row (the D entries of one output node) or, for
    states [B, T], the batch item's T states. The rms term is the floor for elements that
    cancel to near zero; every other element is held to rtol of its own magnitude."""
    g = np.asarray(gpu, np.float64)
    r = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(r * r, axis=-1, keepdims=True))
    scale = np.maximum(np.abs(r) + rms, 1e-6)
    err = np.abs(g - r) / scale
    if g.ndim == 2:  # state [B, T]
        err = err[..., None]
    if skip_rows is not None:
        err = err[~skip_rows]
    worst = float(err.max()) if err.size else 0.0
    assert worst <= rtol, f"{what}: worst relative error {worst:.3e} > {rtol}"
