"""CPU oracle for the Jakal-Net operator hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in NumPy (float64 accumulation), the reference algorithms of the
path the B200 library implements, so that tests, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg of ``bench.py`` can check / time the CUDA kernels against it. It is
never imported by the product package (``jakal_net_b200``), which fails loudly when its
CUDA library is missing instead of falling back to this code.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against
fixtures produced by running the reference implementation itself
(``tests/golden/make_golden.py`` imports Ahnd6474/Jakal-Net in the build container) and
against the reference's own known-answer tests.

Reference citations are ``path:line`` inside the Jakal-Net project.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "round_to",
    "lowrank_project",
    "lowrank_scores",
    "multihead_scores",
    "causal_window_visible",
    "select_topk",
    "compress",
    "entmax15",
    "signed_entmax15",
    "topk_from_scores",
    "masked_dense_from_scores",
    "sparse_transition_from_logits",
    "dense_transition_from_logits",
    "propagation_topk",
    "propagation_masked_dense",
    "transition_pairwise_topk",
    "transition_query_topk",
    "transition_dense",
    "softplus",
]


# ----------------------------------------------------------------------------- rounding
def _round_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even into bfloat16, returned as float32 values."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    nan = np.isnan(f)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    out[nan] = np.nan
    return out


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Value of ``x`` after a cast to ``dtype`` ('f32' | 'bf16' | 'f16'), as float32."""
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return _round_bf16(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)
    raise ValueError(dtype)


def softplus(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.softplus (beta=1, threshold=20)."""
    x = np.asarray(x, dtype=np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


# ----------------------------------------------------------------------------- scores
def lowrank_project(x, w, core=None, temperature: float = 1.0, dtype: str = "bf16") -> np.ndarray:
    """Low-rank projection with the reference's rounding points.

    native/jakal_net_native.cpp:6236-6239: ``projected = matmul(val, W^T)`` in the input
    dtype, ``weighted = projected * w.to(dtype)``; :6979-6983 routes additionally divide
    by the temperature in that dtype. x [..., D], w [R, D], core [R].
    """
    acc = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    out = round_to(acc, dtype)
    if core is not None:
        out = round_to(out.astype(np.float64) * round_to(core, dtype).astype(np.float64), dtype)
    if temperature != 1.0:
        out = round_to(out.astype(np.float64) / float(temperature), dtype)
    return out


def lowrank_scores(row_proj, col_proj, bias: float = 0.0) -> np.ndarray:
    """score[b, t, s] = row_proj[b, t] . col_proj[b, s] + bias  (modules.py:93-100)."""
    return np.einsum("btr,bsr->bts", np.asarray(row_proj, np.float64), np.asarray(col_proj, np.float64)) + bias


def multihead_scores(row_proj, col_proj, head_bias=None, combine: str = "max") -> np.ndarray:
    """MultiHeadPairwise scores (modules.py:274-299): per-head s_h = row_proj[:, h] .
    col_proj[:, h] + bias[h] for row_proj [B, H, T, R], col_proj [B, H, S, R] (core applied),
    combined over the heads: max (:291-298); smoothmax = logsumexp - log H (:276-280);
    signed_smoothmax = sum_h s_h softmax_h(|s_h|) (:281-284). Returns [B, T, S]."""
    s = np.einsum("bhtr,bhsr->bhts", np.asarray(row_proj, np.float64), np.asarray(col_proj, np.float64))
    H = s.shape[1]
    if head_bias is not None:
        s = s + np.asarray(head_bias, np.float64).reshape(1, H, 1, 1)
    if combine == "max":
        return s.max(axis=1)
    if combine == "smoothmax":
        m = s.max(axis=1, keepdims=True)
        return (m + np.log(np.exp(s - m).sum(axis=1, keepdims=True)))[:, 0] - np.log(H)
    if combine == "signed_smoothmax":
        a = np.abs(s)
        w = np.exp(a - a.max(axis=1, keepdims=True))
        w = w / w.sum(axis=1, keepdims=True)
        return (s * w).sum(axis=1)
    raise ValueError(f"unknown head combine {combine!r}")


def causal_window_visible(n_rows: int, n_cols: int, window: int | None) -> np.ndarray:
    """Visibility mask [n_rows, n_cols]; kernel_common.py:443-456 when window is given
    (source <= target and source >= target - window), all-True when window is None."""
    if window is None or window < 0:
        return np.ones((n_rows, n_cols), dtype=bool)
    t = np.arange(n_rows)[:, None]
    s = np.arange(n_cols)[None, :]
    return (s <= t) & (s >= t - window)


def select_topk(scores_row: np.ndarray, visible_row: np.ndarray, k: int) -> np.ndarray:
    """Indices of the min(k, #visible) visible columns with the largest score, ordered by
    (score descending, index ascending). kernel_common.py:426-440 (torch.topk) with the
    tie order fixed to "lower index first"."""
    idx = np.nonzero(visible_row)[0]
    if idx.size == 0:
        return idx
    order = np.lexsort((idx, -scores_row[idx]))
    return idx[order[: min(k, idx.size)]]


# ----------------------------------------------------------------------------- compressors
def entmax15(z: np.ndarray) -> np.ndarray:
    """1.5-entmax over the last axis of a 1-D array (kernels.py:155-210 restated:
    shift by max, halve, sort-based threshold tau, square, renormalise)."""
    z = np.asarray(z, np.float64)
    if z.size == 0:
        return z
    shifted = (z - z.max()) / 2.0
    srt = np.sort(shifted)[::-1]
    rho = np.arange(1, srt.size + 1, dtype=np.float64)
    mean = np.cumsum(srt) / rho
    mean_sq = np.cumsum(srt * srt) / rho
    var = rho * (mean_sq - mean * mean)
    delta = np.clip((1.0 - var) / rho, 0.0, None)
    tau = mean - np.sqrt(delta)
    support = max(int(np.sum(tau <= srt)), 1)
    p = np.clip(shifted - tau[support - 1], 0.0, None) ** 2
    den = p.sum()
    return p / max(den, np.finfo(np.float32).eps) if den > 0 else np.zeros_like(p)


def signed_entmax15(s: np.ndarray) -> np.ndarray:
    """sign(s) * entmax15(|s|)  (kernels.py:222-236)."""
    s = np.nan_to_num(np.asarray(s, np.float64))
    return np.sign(s) * entmax15(np.abs(s))


def compress(sel_scores: np.ndarray, name: str) -> np.ndarray:
    """Edge / route compressor over one row's selected (or visible) scores.

    softsign: propagation.py:85 (F.softsign). signed_abs_softmax: propagation.py:74-82 /
    transition.py:53-67 (softmax of |s| over the row, times sign). signed_entmax15:
    kernels.py:222-236. softmax: transition.py:187-194.
    """
    s = np.asarray(sel_scores, np.float64)
    if s.size == 0:
        return s
    if name == "softsign":
        return s / (1.0 + np.abs(s))
    if name == "softmax":
        e = np.exp(s - s.max())
        return e / e.sum()
    if name == "signed_abs_softmax":
        s = np.nan_to_num(s)
        a = np.abs(s)
        e = np.exp(a - a.max())
        return np.sign(s) * e / e.sum()
    if name == "signed_entmax15":
        return signed_entmax15(s)
    raise ValueError(f"unknown compressor {name!r}")


# ----------------------------------------------------------------------------- operators
def topk_from_scores(scores, col_state, col_val, k: int, *, window: int | None = None, bias: float = 0.0,
                     compress_name: str = "softsign", col_sender=None):
    """Top-k propagation / per-query transition on a given score tensor [B, T, S] (bias
    not included; added after selection, which leaves the selection unchanged).

    window None: reference SparsePropagation(sparse_type="topk") -- top-k over every source
    (propagation.py:453-480, no causal mask; native kernel jakal_net_native_cuda.cu:1029-1183).
    window >= 0: window-intersect-top-k -- causal_window_mask (kernel_common.py:443-456),
    top-k among the visible sources, edges over the survivors.
    col_sender (per-query transition, jakal_net_native.cpp:7221-7246): edges are
    multiplied by the sender strength of the picked source.
    Returns (state [B,T], val [B,T,D], sel_scores [B,T,k] (-inf pad), sel_index [B,T,k] (-1 pad)).
    """
    sc = np.asarray(scores, np.float64)
    B, T, S = sc.shape
    vis = causal_window_visible(T, S, window)
    st = np.asarray(col_state, np.float64)
    val = np.asarray(col_val, np.float64)
    snd = None if col_sender is None else np.asarray(col_sender, np.float64)
    out_state = np.zeros((B, T))
    out_val = np.zeros((B, T, val.shape[-1]))
    sel_scores = np.full((B, T, k), -np.inf)
    sel_index = np.full((B, T, k), -1, dtype=np.int64)
    for b in range(B):
        for t in range(T):
            idx = select_topk(sc[b, t], vis[t], k)
            if idx.size == 0:
                continue
            s = sc[b, t, idx] + bias
            sel_scores[b, t, : idx.size] = s
            sel_index[b, t, : idx.size] = idx
            e = compress(s, compress_name)
            if snd is not None:
                e = e * snd[b, idx]
            out_state[b, t] = e @ st[b, idx]
            out_val[b, t] = e @ val[b, idx]
    return out_state, out_val, sel_scores, sel_index


def propagation_topk(row_proj, col_proj, col_state, col_val, k: int, *, window: int | None = None,
                     bias: float = 0.0, compress_name: str = "softsign", col_sender=None):
    """topk_from_scores on the low-rank scores row_proj . col_proj (modules.py:93-100)."""
    return topk_from_scores(lowrank_scores(row_proj, col_proj, 0.0), col_state, col_val, k, window=window,
                            bias=bias, compress_name=compress_name, col_sender=col_sender)


def masked_dense_from_scores(scores, col_state, col_val, *, window: int | None, compress_name: str = "softsign"):
    """Dense (window None) or causal-window propagation without top-k on a score tensor
    (bias included): propagation.py:207-220 (dense) and :453-480 with the window mask; edges
    are compressed over each row's visible sources (propagation.py:67-88), masked entries
    contribute 0."""
    sc = np.asarray(scores, np.float64)
    B, T, S = sc.shape
    vis = causal_window_visible(T, S, window)
    st = np.asarray(col_state, np.float64)
    val = np.asarray(col_val, np.float64)
    out_state = np.zeros((B, T))
    out_val = np.zeros((B, T, val.shape[-1]))
    for t in range(T):
        idx = np.nonzero(vis[t])[0]
        if idx.size == 0:
            continue
        for b in range(B):
            e = compress(sc[b, t, idx], compress_name)
            out_state[b, t] = e @ st[b, idx]
            out_val[b, t] = e @ val[b, idx]
    return out_state, out_val


def propagation_masked_dense(row_proj, col_proj, col_state, col_val, *, window: int | None,
                             bias: float = 0.0, compress_name: str = "softsign"):
    """masked_dense_from_scores on the low-rank scores."""
    return masked_dense_from_scores(lowrank_scores(row_proj, col_proj, bias), col_state, col_val, window=window,
                                    compress_name=compress_name)


def sparse_transition_from_logits(logits, src_state, src_val, src_sender, k: int, *, compress_name: str = "softmax"):
    """Per-source sparse transition on route logits [B, S, Dn] (bias included)
    (SparseTransition, transition.py:431-452 / 483-590; native jakal_net_native.cpp:6916-7087):
    every source picks its top-k destinations, routes are compressed over those k, weighted
    by the sender strength and scatter-added into the destinations."""
    lg = np.asarray(logits, np.float64)
    B, S, Dn = lg.shape
    st = np.asarray(src_state, np.float64)
    val = np.asarray(src_val, np.float64)
    snd = np.asarray(src_sender, np.float64)
    out_state = np.zeros((B, Dn))
    out_val = np.zeros((B, Dn, val.shape[-1]))
    allv = np.ones(Dn, dtype=bool)
    for b in range(B):
        for i in range(S):
            idx = select_topk(lg[b, i], allv, k)
            r = compress(lg[b, i, idx], compress_name) * snd[b, i]
            np.add.at(out_state[b], idx, r * st[b, i])
            out_val[b, idx] += r[:, None] * val[b, i][None, :]
    return out_state, out_val


def transition_pairwise_topk(src_proj, dst_proj, src_state, src_val, src_sender, k: int, *,
                             bias: float = 0.0, compress_name: str = "softmax"):
    """sparse_transition_from_logits on the low-rank route logits."""
    return sparse_transition_from_logits(lowrank_scores(src_proj, dst_proj, bias), src_state, src_val, src_sender, k,
                                         compress_name=compress_name)


def transition_query_topk(query_proj, source_proj, src_state, src_val, src_sender, k: int, *,
                          bias: float = 0.0):
    """Per-query transition (jakal_net_native.cpp:7089-7246): every query slot picks its
    top-k sources by route logit route(src, query)^T, softmax over the k, and gathers
    softplus-weighted source state / value."""
    return propagation_topk(query_proj, source_proj, src_state, src_val, k, window=None, bias=bias,
                            compress_name="softmax", col_sender=src_sender)


def dense_transition_from_logits(logits, src_state, src_val, src_sender, *, compress_name: str = "softmax"):
    """Dense transition (transition.py:238-254) on route logits: routes compressed over all
    destinations per source, weighted by the sender strength, summed into every destination."""
    lg = np.asarray(logits, np.float64)
    B, S, Dn = lg.shape
    st = np.asarray(src_state, np.float64)
    val = np.asarray(src_val, np.float64)
    snd = np.asarray(src_sender, np.float64)
    routes = np.zeros_like(lg)
    for b in range(B):
        for i in range(S):
            routes[b, i] = compress(lg[b, i], compress_name) * snd[b, i]
    return np.einsum("bsd,bs->bd", routes, st), np.einsum("bsd,bsv->bdv", routes, val)


def transition_dense(src_proj, dst_proj, src_state, src_val, src_sender, *, bias: float = 0.0,
                     compress_name: str = "softmax"):
    """dense_transition_from_logits on the low-rank route logits."""
    return dense_transition_from_logits(lowrank_scores(src_proj, dst_proj, bias), src_state, src_val, src_sender,
                                        compress_name=compress_name)
