"""Multi-threaded CPU port of the reference's blocked CPU path — TEST / BASELINE ONLY.

``bench.py`` times this as the CPU baseline (``cpu_baseline`` and ``--impl reference``):
the reference's own CPU implementation of the path cannot travel to the GPU host (its
source tree is not present there), so this file restates its blocked algorithm in torch
CPU ops, block by block as native/jakal_net_native.cpp:6305-6447 (top-k) and
:6190-6303 (window) do: per target block, score the visible source block with a matmul of
the low-rank projections, take the top-k (torch.topk), compress the k survivors and
aggregate with a gather. Checked against the loop oracle in tests/test_oracle_cpu.py.

It is never imported by the product package.
"""
from __future__ import annotations

import torch
from torch.nn import functional as F


def _compress(scores: torch.Tensor, name: str) -> torch.Tensor:
    if name == "softsign":
        return F.softsign(scores)
    if name == "softmax":
        return torch.softmax(scores, dim=-1)
    if name == "signed_abs_softmax":
        return torch.sign(scores) * torch.softmax(scores.abs(), dim=-1)
    raise ValueError(name)


@torch.no_grad()
def window_topk_propagation(row_proj: torch.Tensor, col_proj: torch.Tensor, state: torch.Tensor,
                            val: torch.Tensor, k: int, window: int | None, *, bias: float = 0.0,
                            compress: str = "softsign", block: int = 128):
    """Blocked window-intersect-top-k propagation on CPU.

    row_proj / col_proj [B, N, R] float32 (projection values), state [B, N], val [B, N, D].
    window None = top-k over every source (reference SparsePropagation topk semantics).
    Returns (state [B, N], val [B, N, D]) float32. Rows with fewer than k visible sources
    keep all of them (masked slots carry -inf and contribute nothing). Only softsign is
    exact for such short rows (masked slots are excluded from the normalisation of the
    normalising compressors only when every row has at least k visible sources).
    """
    B, N, _ = row_proj.shape
    D = val.shape[-1]
    out_state = torch.zeros(B, N)
    out_val = torch.zeros(B, N, D)
    ar = torch.arange(N)
    for t0 in range(0, N, block):
        t1 = min(N, t0 + block)
        s0 = 0 if window is None else max(0, t0 - window)
        s1 = N if window is None else t1
        sc = torch.matmul(row_proj[:, t0:t1], col_proj[:, s0:s1].transpose(1, 2))  # [B, bt, bs]
        if window is not None:
            t = ar[t0:t1, None]
            s = ar[None, s0:s1]
            vis = (s <= t) & (s >= t - window)
            sc = sc.masked_fill(~vis, float("-inf"))
        kk = min(k, s1 - s0)
        top = torch.topk(sc, kk, dim=-1)
        valid = torch.isfinite(top.values)
        e = _compress(torch.where(valid, top.values + bias, torch.zeros_like(top.values)), compress)
        e = torch.where(valid, e, torch.zeros_like(e))
        idx = top.indices + s0
        g_state = torch.gather(state[:, None, :].expand(B, t1 - t0, N), 2, idx)
        out_state[:, t0:t1] = (e * g_state).sum(-1)
        flat = idx.reshape(B, -1)
        g_val = torch.gather(val, 1, flat[..., None].expand(B, flat.shape[1], D)).reshape(B, t1 - t0, kk, D)
        out_val[:, t0:t1] = torch.einsum("btk,btkd->btd", e, g_val)
    return out_state, out_val


def lowrank_project_bf16(x: torch.Tensor, w: torch.Tensor, core: torch.Tensor | None = None) -> torch.Tensor:
    """torch.matmul in bfloat16 on CPU then the elementwise core multiply in bfloat16
    (jakal_net_native.cpp:6236-6239); returned as float32 values."""
    p = torch.matmul(x.to(torch.bfloat16), w.to(torch.bfloat16).t())
    if core is not None:
        p = p * core.to(torch.bfloat16)
    return p.float()
