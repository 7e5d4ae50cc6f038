"""GPU parity of the fused top-k kernels against the CPU oracle (through the C ABI)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import parity

pytestmark = pytest.mark.gpu


def _jk():
    import jakal_net_b200 as jk
    return jk


def _bf16(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev).to(torch.bfloat16)


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _make(B, N, D, R, seed, dev, n_cols=None):
    g = np.random.default_rng(seed)
    S = N if n_cols is None else n_cols
    val_rows = g.standard_normal((B, N, D)).astype(np.float32)
    val_cols = val_rows if n_cols is None else g.standard_normal((B, S, D)).astype(np.float32)
    state = g.standard_normal((B, S)).astype(np.float32)
    wt = (g.standard_normal((R, D)) / np.sqrt(D)).astype(np.float32)
    ws = (g.standard_normal((R, D)) / np.sqrt(D)).astype(np.float32)
    core = np.full(R, 1.0 / np.sqrt(R), np.float32)
    return dict(val_rows=_bf16(val_rows, dev), val_cols=_bf16(val_cols, dev), state=_bf16(state, dev),
                wt=_bf16(wt, dev), ws=_bf16(ws, dev), core=_bf16(core, dev))


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("rows,dim,rank", [(300, 64, 64), (1000, 384, 64), (257, 128, 96)])
def test_projection_matches_oracle(dev, rows, dim, rank):
    jk = _jk()
    g = np.random.default_rng(rows)
    x = _bf16(g.standard_normal((rows, dim)), dev)
    w = _bf16(g.standard_normal((rank, dim)) / np.sqrt(dim), dev)
    core = _bf16(np.linspace(0.05, 0.2, rank), dev)
    for c, temp in ((None, 1.0), (core, 1.0), (core, 0.7)):
        out = jk.lowrank_project(x, w, core=c, temperature=temp)
        torch.cuda.synchronize()
        rp = out.shape[-1]
        assert rp == ((rank + 63) // 64) * 64
        got = _np(out)
        ref = oracle.lowrank_project(_np(x), _np(w), None if c is None else _np(c), temp, "bf16")
        assert np.all(got[:, rank:] == 0)
        # f32 accumulation order differs from the float64 oracle: allow rare 1-ulp flips.
        diff = got[:, :rank] != ref
        assert diff.mean() < 2e-3, f"{diff.mean():.2e} of projections differ"
        # A flip is one rounding step of the (near-identical) f32 sum, which the later
        # multiply / divide roundings can carry into up to a few final ulps (2^-6 relative),
        # or tiny in absolute terms where the dot product cancels to ~0.
        err = np.abs(got[:, :rank] - ref)
        scale = 1.0 if c is None else np.abs(_np(c))[None, :] / temp
        bad = err > 2 ** -6 * np.abs(ref) + 2e-5 * scale
        assert not bad.any(), (err[bad][:5], ref[bad][:5], got[:, :rank][bad][:5])


def _check_topk(dev, B, N, D, R, k, window, compress_name, seed, n_cols=None, sender=False):
    jk = _jk()
    d = _make(B, N, D, R, seed, dev, n_cols)
    row_proj = jk.lowrank_project(d["val_rows"], d["wt"])
    col_proj = jk.lowrank_project(d["val_cols"], d["ws"], core=d["core"])
    snd = torch.nn.functional.softplus(d["state"].float()).to(torch.bfloat16) if sender else None
    code = {"softsign": 0, "signed_abs_softmax": 1, "signed_entmax15": 2, "softmax": 3}[compress_name]
    bias = torch.tensor([0.125], device=dev)
    st, vv, sc, ix = jk.topk_aggregate(row_proj, col_proj, d["state"], d["val_cols"], k, window=window,
                                       compress=code, col_sender=snd, bias=bias, out_dtype=torch.float32,
                                       return_selection=True)
    torch.cuda.synchronize()
    rp_ = _np(row_proj)
    cp_ = _np(col_proj)
    o_st, o_val, o_sc, o_ix = oracle.propagation_topk(
        rp_, cp_, _np(d["state"]), _np(d["val_cols"]), k, window=None if window < 0 else window, bias=0.125,
        compress_name=compress_name, col_sender=None if snd is None else _np(snd))
    full = oracle.lowrank_scores(rp_, cp_, 0.125)
    parity.set_full_scores(full)
    ties = parity.tie_rows(_np(ix).astype(np.int64), o_ix, o_sc)
    assert ties.mean() < 0.01, f"too many tie rows: {ties.mean():.3%}"
    ok = ~ties
    np.testing.assert_allclose(_np(sc)[ok], o_sc[ok], rtol=1e-5, atol=1e-5)
    parity.assert_rows_close(_np(vv), o_val, ties, what="val")
    parity.assert_rows_close(_np(st), o_st, ties, what="state")


@pytest.mark.parametrize("compress_name", ["softsign", "signed_abs_softmax", "signed_entmax15", "softmax"])
def test_topk_all_sources(dev, compress_name):
    _check_topk(dev, B=2, N=300, D=64, R=64, k=8, window=-1, compress_name=compress_name, seed=1)


@pytest.mark.parametrize("window,k", [(0, 4), (5, 8), (50, 8), (200, 32), (299, 64)])
def test_topk_window(dev, window, k):
    _check_topk(dev, B=2, N=300, D=64, R=64, k=k, window=window, compress_name="softsign", seed=2)


def test_topk_query_transition_shape(dev):
    _check_topk(dev, B=2, N=130, D=128, R=64, k=16, window=-1, compress_name="softmax", seed=3, n_cols=700,
                sender=True)


def test_topk_config2_reduced(dev):
    _check_topk(dev, B=1, N=2048, D=384, R=64, k=32, window=512, compress_name="softsign", seed=4)


def test_topk_rank_128(dev):
    _check_topk(dev, B=1, N=400, D=64, R=100, k=16, window=-1, compress_name="softsign", seed=5)


def _check_given(dev, val_rows, k, window, compress_name="softsign", seed=0):
    """Parity on caller-shaped inputs (exercises the threshold fallback path)."""
    jk = _jk()
    g = np.random.default_rng(seed)
    B, N, D = val_rows.shape
    R = 64
    val = _bf16(val_rows, dev)
    state = _bf16(g.standard_normal((B, N)), dev)
    wt = _bf16(g.standard_normal((R, D)) / np.sqrt(D), dev)
    ws = _bf16(g.standard_normal((R, D)) / np.sqrt(D), dev)
    core = _bf16(np.full(R, 1.0 / np.sqrt(R)), dev)
    row_proj = jk.lowrank_project(val, wt)
    col_proj = jk.lowrank_project(val, ws, core=core)
    code = {"softsign": 0, "signed_abs_softmax": 1, "signed_entmax15": 2, "softmax": 3}[compress_name]
    st, vv, sc, ix = jk.topk_aggregate(row_proj, col_proj, state, val, k, window=window, compress=code,
                                       out_dtype=torch.float32, return_selection=True)
    torch.cuda.synchronize()
    rp_, cp_ = _np(row_proj), _np(col_proj)
    o_st, o_val, o_sc, o_ix = oracle.propagation_topk(rp_, cp_, _np(state), _np(val), k,
                                                      window=None if window < 0 else window,
                                                      compress_name=compress_name)
    parity.set_full_scores(oracle.lowrank_scores(rp_, cp_, 0.0))
    ties = parity.tie_rows(_np(ix).astype(np.int64), o_ix, o_sc)
    parity.assert_rows_close(_np(vv), o_val, ties, what="val")
    parity.assert_rows_close(_np(st), o_st, ties, what="state")
    return ties


def test_topk_all_equal_scores_fallback(dev):
    # Every row identical -> every score equal: the threshold pass overflows, the exact
    # fallback keeps the k lowest columns (ties to the lower index).
    row = np.random.default_rng(7).standard_normal((1, 1, 64))
    val = np.repeat(row, 600, axis=1)
    _check_given(dev, val, k=16, window=-1)
    _check_given(dev, val, k=32, window=300)


def test_topk_bimodal_scores(dev):
    # Two clusters of rows far apart: strongly non-normal score rows.
    g = np.random.default_rng(8)
    val = g.standard_normal((2, 700, 64))
    val[:, ::7] *= 12.0
    ties = _check_given(dev, val, k=32, window=-1)
    assert ties.mean() < 0.05


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rank,core,temperature", [(64, True, 1.0), (40, True, 0.7), (17, False, 1.0)])
def test_pair_projection_equals_two_projections(dev, dtype, rank, core, temperature):
    import jakal_net_b200 as jk

    g = torch.Generator().manual_seed(rank)
    rows, dim = 1000, 192
    x = torch.randn(rows, dim, generator=g).to(dev, dtype)
    w = (torch.randn(rank, dim, generator=g) / dim ** 0.5).to(dev, dtype)
    w2 = (torch.randn(rank, dim, generator=g) / dim ** 0.5).to(dev, dtype)
    c = (torch.rand(rank, generator=g) + 0.5).to(dev, dtype) if core else None
    a, b = jk.lowrank_project_pair(x, w, w2, core=c, temperature=temperature)
    assert torch.equal(a, jk.lowrank_project(x, w))
    assert torch.equal(b, jk.lowrank_project(x, w2, core=c, temperature=temperature))
