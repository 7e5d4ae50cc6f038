"""Query-row-block sharding of a causal-window top-k propagation over the GPUs of one node.

A long causal window (benchmark configuration 5: B4, N32768, window 4096, k 64) does not
split by batch item across 8 GPUs, so the target rows are split instead: rank r owns the
row block [r * blk, (r + 1) * blk) (whole 128-row tiles). Its rows only read source rows
[begin - window, begin + blk), but the inputs are kept replicated on every GPU (one
broadcast at setup), so every rank calls the fused kernel on the full tensors and computes
only its block (jk_propagation_topk_rows_forward). The output blocks are then assembled on
every rank by an all-gather -- the only collective, and only where a caller needs the full
result on every GPU (the next layer can consume the row-sharded outputs directly).

This module is host-side plumbing over torch.distributed (NCCL on GPUs, gloo in the CPU
tests); the per-rank compute is the library's kernel unless a test passes `block_fn`.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist
from torch import Tensor

TILE = 128  # rows per CTA of the fused kernel: row blocks start on tile boundaries


def row_blocks(n_rows: int, world: int, tile: int = TILE) -> list[tuple[int, int]]:
    """(begin, count) of every rank's row block: equal whole-tile blocks, the last one
    clipped to n_rows (count 0 for ranks beyond the last tile)."""
    if n_rows <= 0 or world <= 0:
        raise ValueError("n_rows and world must be positive")
    tiles = -(-n_rows // tile)
    per = -(-tiles // world) * tile
    out = []
    for r in range(world):
        b = min(r * per, n_rows)
        out.append((b, min(b + per, n_rows) - b))
    return out


def replicate(t: Tensor, src: int = 0, group=None) -> Tensor:
    """Makes `t` identical on every rank (broadcast from `src`, in place)."""
    dist.broadcast(t, src=src, group=group)
    return t


def _kernel_block(row_proj, col_proj, col_state, col_val, k, window, begin, count, out_state, out_val, **kw):
    from . import check, _LIBRARY, _dtype_code, _proj_dtype, _ptr, _stream

    B, N, rp = row_proj.shape
    S = col_proj.shape[1]
    D = col_val.shape[-1]
    dev = col_val.device
    bias = kw.get("bias")
    with torch.cuda.device(dev):
        check(
            _LIBRARY.jk_propagation_topk_rows_forward(
                row_proj.data_ptr(), col_proj.data_ptr(), B, N, begin, count, S, rp, _proj_dtype(row_proj),
                col_state.data_ptr(), None, _dtype_code("state", col_state), col_val.data_ptr(), D,
                _dtype_code("val", col_val), k, window, float(kw.get("score_bias", 0.0)), _ptr(bias),
                kw.get("compress", 0), out_state.data_ptr(), out_val.data_ptr(), _dtype_code("out", out_state),
                None, None, _stream(dev)),
            "jk_propagation_topk_rows_forward",
        )


def gather_row_blocks(out_state: Tensor, out_val: Tensor, blocks: list[tuple[int, int]], group=None,
                      stream: Optional[torch.cuda.Stream] = None):
    """Assembles the row blocks every rank wrote into its own out_state [B, N] / out_val
    [B, N, D] so that every rank holds the full outputs. Equal blocks that tile the rows (the
    usual case) are gathered in place, one all-gather per batch item and tensor, with no
    copies; otherwise one rank-major all-gather per tensor (the rank's block of every batch
    item packed into a [B, blk, ...] buffer, gathered into [world, B, blk, ...]) -- two
    collectives whatever the batch size -- then the blocks are copied into place. With `stream` the exchange runs on that stream
    (ordered after the current stream's work), so a caller can overlap it with compute."""
    world = len(blocks)
    rank = dist.get_rank(group)
    blk = max(c for _, c in blocks)
    B = out_state.shape[0]
    begin, count = blocks[rank]
    ctx = torch.cuda.stream(stream) if stream is not None else _nullcontext()
    if stream is not None:
        stream.wait_stream(torch.cuda.current_stream(out_val.device))
    with ctx:
        if all(c == blk and b0 == r * blk for r, (b0, c) in enumerate(blocks)):
            # equal blocks tiling the rows: every batch item's rows are already rank-major,
            # so each item is gathered in place (the rank's block is the input, the whole
            # item the output) -- no packing or unpacking copies
            for full in (out_state, out_val):
                for b in range(B):
                    item = full[b]
                    dist.all_gather_into_tensor(item.view(-1), item[begin:begin + count].reshape(-1), group=group)
            return out_state, out_val
        for full in (out_state, out_val):
            send = full.new_zeros((B, blk) + tuple(full.shape[2:]))
            send[:, :count] = full[:, begin:begin + count]
            recv = full.new_empty((world * B,) + tuple(send.shape[1:]))  # rank-major concatenation
            dist.all_gather_into_tensor(recv, send, group=group)
            recv = recv.view((world,) + tuple(send.shape))
            for r, (b0, c) in enumerate(blocks):
                if c:
                    full[:, b0:b0 + c] = recv[r, :, :c]
    return out_state, out_val


class _nullcontext:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def propagation_window_topk_rows(row_proj: Tensor, col_proj: Tensor, col_state: Tensor, col_val: Tensor, k: int,
                                 window: int, *, group=None, gather: bool = True, out_dtype=None,
                                 block_fn: Optional[Callable] = None, **kernel_kw):
    """Row-sharded window-intersect-top-k propagation over already-projected, replicated
    inputs (row_proj [B, N, rp], col_proj [B, N, rp], col_state [B, N], col_val [B, N, D]).
    Every rank computes its row block; with gather=True the full (state [B, N], val
    [B, N, D]) is returned on every rank, else the rank's outputs with only its block
    written, and its (begin, count)."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    B, N, _ = row_proj.shape
    D = col_val.shape[-1]
    blocks = row_blocks(N, world)
    begin, count = blocks[rank]
    dt = out_dtype or col_val.dtype
    out_state = torch.zeros((B, N), device=col_val.device, dtype=dt)
    out_val = torch.zeros((B, N, D), device=col_val.device, dtype=dt)
    if count > 0:
        (block_fn or _kernel_block)(row_proj, col_proj, col_state, col_val, k, window, begin, count, out_state,
                                    out_val, **kernel_kw)
    if not gather:
        return out_state, out_val, (begin, count)
    gather_row_blocks(out_state, out_val, blocks, group)
    return out_state, out_val
