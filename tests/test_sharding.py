"""Row-block sharding (jakal_net_b200.sharding): the partition, and the multi-rank
assembly run as two gloo ranks on the CPU, each rank's block computed by the CPU oracle
(the per-rank step the GPU kernel performs; its own parity is tests/test_gpu_rows.py)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from jakal_net_b200.sharding import propagation_window_topk_rows, row_blocks


def test_row_blocks_cover_rows_once_on_tile_boundaries():
    for n, w in [(32768, 8), (1000, 3), (129, 2), (100, 4), (5000, 7)]:
        blocks = row_blocks(n, w)
        assert len(blocks) == w
        covered = np.zeros(n, int)
        for b, c in blocks:
            assert b % 128 == 0 or c == 0
            covered[b:b + c] += 1
        assert (covered == 1).all()
    assert row_blocks(32768, 8) == [(4096 * r, 4096) for r in range(8)]


def _inputs(B, N, D, R):
    g = np.random.default_rng(12)
    pt = g.standard_normal((B, N, R)).astype(np.float32)
    ps = g.standard_normal((B, N, R)).astype(np.float32)
    st = g.standard_normal((B, N)).astype(np.float32)
    val = g.standard_normal((B, N, D)).astype(np.float32)
    return pt, ps, st, val


def _oracle_block(row_proj, col_proj, col_state, col_val, k, window, begin, count, out_state, out_val, **kw):
    # rows [begin, begin + count) of the full problem, with the oracle's own window semantics
    # (it indexes rows from 0, so it runs on rows [0, begin + count) and keeps the block)
    sc = oracle.lowrank_scores(row_proj[:, :begin + count].numpy(), col_proj.numpy())
    st, val, _, _ = oracle.topk_from_scores(sc, col_state.numpy(), col_val.numpy(), k, window=window)
    out_state[:, begin:begin + count] = torch.from_numpy(st[:, begin:].astype(np.float32))
    out_val[:, begin:begin + count] = torch.from_numpy(val[:, begin:].astype(np.float32))


def _rank_main(rank, world, port, shape, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, N, D, R, k, W = shape
        pt, ps, st, val = (torch.from_numpy(a) for a in _inputs(B, N, D, R))
        s, v = propagation_window_topk_rows(pt, ps, st, val, k, W, block_fn=_oracle_block, out_dtype=torch.float32)
        result_q.put((rank, s.numpy(), v.numpy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("shape", [(2, 512, 8, 4, 5, 100), (2, 300, 8, 4, 3, 77)])
def test_row_sharded_assembly_matches_unsharded_gloo(shape):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, shape, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    B, N, D, R, k, W = shape
    pt, ps, st, val = _inputs(B, N, D, R)
    ref_s, ref_v, _, _ = oracle.topk_from_scores(oracle.lowrank_scores(pt, ps), st, val, k, window=W)
    for _, s, v in results:
        np.testing.assert_allclose(s, ref_s, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(v, ref_v, rtol=1e-5, atol=1e-5)
