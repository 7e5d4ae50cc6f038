"""Row blocks of the fused top-k kernel (jk_propagation_topk_rows_forward, the per-rank step
of the row-sharded multi-GPU propagation): stitched blocks reproduce the single launch bit
for bit (same 128-row CTAs, same arithmetic), and misaligned blocks are rejected."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("shape", [(2, 1100, 128, 300, 16, 3), (1, 2048, 384, 512, 32, 4), (2, 700, 64, -1, 8, 2)])
def test_stitched_row_blocks_equal_the_full_launch(dev, shape):
    import jakal_net_b200 as jk
    from jakal_net_b200.sharding import row_blocks

    B, N, D, W, k, world = shape
    g = torch.Generator().manual_seed(N + D)
    val = torch.randn(B, N, D, generator=g).to(dev, torch.bfloat16)
    state = torch.randn(B, N, generator=g).to(dev, torch.bfloat16)
    rp = (torch.randn(B, N, 64, generator=g) / 8).to(dev, torch.bfloat16)
    cp = (torch.randn(B, N, 64, generator=g) / 8).to(dev, torch.bfloat16)
    full_s, full_v = jk.topk_aggregate(rp, cp, state, val, k, window=W)
    got_s = torch.zeros_like(full_s)
    got_v = torch.zeros_like(full_v)
    for begin, count in row_blocks(N, world):
        if count == 0:
            continue
        s, v = jk.topk_aggregate(rp, cp, state, val, k, window=W, rows=(begin, count))
        got_s[:, begin:begin + count] = s[:, begin:begin + count]
        got_v[:, begin:begin + count] = v[:, begin:begin + count]
        # rows outside the block are left untouched
        assert not s[:, :begin].any() and not s[:, begin + count:].any()
    assert torch.equal(got_s, full_s)
    assert torch.equal(got_v, full_v)


@pytest.mark.parametrize("rows", [(64, 256), (0, 100), (128, 2000), (-128, 128)])
def test_misaligned_row_blocks_are_rejected(dev, rows):
    import jakal_net_b200 as jk

    B, N, D = 1, 1024, 64
    val = torch.randn(B, N, D, device=dev).to(torch.bfloat16)
    state = torch.randn(B, N, device=dev).to(torch.bfloat16)
    rp = torch.randn(B, N, 64, device=dev).to(torch.bfloat16)
    with pytest.raises(jk.JakalB200Error):
        jk.topk_aggregate(rp, rp, state, val, 4, window=100, rows=rows)
