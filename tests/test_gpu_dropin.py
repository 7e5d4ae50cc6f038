"""The drop-in proof: the reference's own Layer API, loader and Progressive-B model running on
this backend.

The staged reference package (baseline/_ref, made by baseline/stage_reference.py) is
imported and its loader is pointed at this module with JAKAL_NET_NATIVE_MODULE=jakal_net_b200
(native_backend.py:33-34, 98-160). Every case follows the reference's own CUDA backend tests
(tests/test_native_backend.py:214-1007): the operator runs once with
implementation="reference" and once with implementation="native"; the module op is wrapped
with mock.patch.object(..., wraps=...) to prove the native call happened, and the deltas are
compared. f32 inputs: the reference's tolerance (1e-5 absolute and relative). The
Progressive-B query-block forward (scripts/progressive_b_example.py:2059) runs end to end on
the backend at a reduced size of config 4's architecture."""
from __future__ import annotations

import contextlib
import os
import sys
from pathlib import Path
from unittest import mock

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "baseline"))
import reference_shim  # noqa: E402  (baseline/reference_shim.py)

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not reference_shim.available(),
                       reason="reference not staged (python baseline/stage_reference.py)"),
]


@pytest.fixture(scope="module")
def jn():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    os.environ["JAKAL_NET_NATIVE_MODULE"] = "jakal_net_b200"
    pkg = reference_shim.import_reference()
    status = pkg.native_status(force_reload=True)
    assert status.available, status.error
    assert status.backend_name == "b200_sm100a" and "cuda" in status.supported_devices
    yield pkg
    pkg.native_status(force_reload=True)


@pytest.fixture(scope="module")
def module(jn):
    import jakal_net.native_backend as nb

    mod = nb._native_module()
    assert mod.__name__ == "jakal_net_b200"
    return mod


def _state_proj(state):
    return state * 1.25 - 0.5


def _val_proj(val):
    return val * 0.5 + 0.25


def signed_abs_softmax_edges(scores):
    """sign(s) * softmax(|s|); the reference's dispatch recognises the edge compressor by
    this function name (propagation.py:56-64)."""
    clean = torch.nan_to_num(scores)
    return torch.sign(clean) * torch.softmax(clean.abs(), dim=-1)


def signed_entmax15(scores):
    """The reference's signed_entmax15 edges (kernels.py:155-236), recognised by name."""
    from jakal_net.kernels import signed_entmax15 as ref_entmax

    return ref_entmax(scores, dim=-1)


def _close(a, b, atol=1e-5, rtol=1e-5):
    assert torch.allclose(a.delta_state, b.delta_state, atol=atol, rtol=rtol), \
        (a.delta_state - b.delta_state).abs().max()
    assert torch.allclose(a.delta_val, b.delta_val, atol=atol, rtol=rtol), (a.delta_val - b.delta_val).abs().max()


def _pair(make, **kw):
    ref = make(implementation="reference", **kw)
    nat = make(implementation="native", **kw)
    nat.load_state_dict(ref.state_dict())
    return ref, nat


def _layer(jn, n, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return jn.Layer(dim=d, num_nodes=n, state=torch.randn(2, n, device="cuda", generator=g),
                    val=torch.randn(2, n, d, device="cuda", generator=g))


def test_dense_propagation_diagonal(jn, module):
    layer = _layer(jn, 7, 4, 30)
    pw = jn.DiagonalBilinearPairwise(dim=4).cuda()
    ref, nat = _pair(lambda **kw: jn.Propagation(pairwise_fn=pw, state_proj_fn=_state_proj, val_proj_fn=_val_proj,
                                                 **kw))
    with mock.patch.object(module, "propagation_dense", wraps=module.propagation_dense) as w:
        got = nat.compute_delta(layer)
    assert w.call_count > 0
    _close(ref.compute_delta(layer), got)


def test_dense_propagation_low_rank_signed_abs_state_weighted(jn, module):
    layer = _layer(jn, 6, 4, 302)
    pw = jn.LowRankBilinearPairwise(dim=4, rank=3).cuda()
    ref, nat = _pair(lambda **kw: jn.Propagation(pairwise_fn=pw, edge_compress_fn=signed_abs_softmax_edges,
                                                 state_proj_fn=_state_proj, val_proj_fn=_val_proj,
                                                 state_weight_edges=True, **kw))
    with mock.patch.object(module, "propagation_dense", wraps=module.propagation_dense) as w:
        got = nat.compute_delta(layer)
    assert w.call_count > 0
    _close(ref.compute_delta(layer), got)


def test_sparse_propagation_window_and_topk(jn, module):
    layer = _layer(jn, 9, 5, 31)
    pw = jn.DiagonalBilinearPairwise(dim=5).cuda()
    ref, nat = _pair(lambda **kw: jn.SparsePropagation(pairwise_fn=pw, state_proj_fn=_state_proj,
                                                       val_proj_fn=_val_proj, sparse_type="window", window=3, **kw))
    with mock.patch.object(module, "propagation_window", wraps=module.propagation_window) as w:
        got = nat.compute_delta(layer)
    assert w.call_count > 0
    _close(ref.compute_delta(layer), got)

    full = jn.BilinearPairwise(dim=5).cuda()
    ref, nat = _pair(lambda **kw: jn.SparsePropagation(pairwise_fn=full, state_proj_fn=_state_proj,
                                                       val_proj_fn=_val_proj, sparse_type="topk", topk=3, **kw))
    with mock.patch.object(module, "propagation_topk", wraps=module.propagation_topk) as w:
        got = nat.compute_delta(layer)
    assert w.call_count > 0
    _close(ref.compute_delta(layer), got)


@pytest.mark.parametrize("edge", ["softsign", "signed_abs", "signed_entmax15"])
@pytest.mark.parametrize("k", [3, 65, 200])
def test_sparse_propagation_topk_any_k(jn, module, edge, k):
    """k beyond the reference CUDA kernels' 64 (they fall back to the blocked path,
    jakal_net_native.cpp:6390-6447); here the select-aggregate kernel takes it."""
    layer = _layer(jn, 300, 24, 40 + k)
    pw = jn.LowRankBilinearPairwise(dim=24, rank=16).cuda()
    kw = {"softsign": {}, "signed_abs": {"edge_compress_fn": signed_abs_softmax_edges},
          "signed_entmax15": {"edge_compress_fn": signed_entmax15}}[edge]
    ref, nat = _pair(lambda **a: jn.SparsePropagation(pairwise_fn=pw, sparse_type="topk", topk=k, **kw, **a))
    with mock.patch.object(module, "propagation_topk", wraps=module.propagation_topk) as w:
        got = nat.compute_delta(layer)
    assert w.call_count > 0
    _close(ref.compute_delta(layer), got, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("route", ["diagonal", "low_rank"])
@pytest.mark.parametrize("compress", ["softmax", "signed_abs_softmax"])
def test_dense_transition_pairwise_routes(jn, module, route, compress):
    src = _layer(jn, 7, 4, 320)
    dst = _layer(jn, 6, 4, 321)
    make_route = (lambda: jn.DiagonalBilinearRoute(src_dim=4, dst_dim=4)) if route == "diagonal" else \
        (lambda: jn.LowRankBilinearRoute(src_dim=4, dst_dim=4, rank=3))
    rf = make_route().cuda()
    ref, nat = _pair(lambda **kw: jn.Transition(route_fn=rf, route_compress_name=compress,
                                                state_activation_fn=lambda x: x + 1.25, val_proj_fn=_val_proj,
                                                state_proj_fn=_state_proj, **kw))
    with mock.patch.object(module, "transition_pairwise_dense", wraps=module.transition_pairwise_dense) as w:
        got = nat.compute_delta(src, dst)
    assert w.call_count > 0
    _close(ref.compute_delta(src, dst), got)


@pytest.mark.parametrize("route", ["diagonal", "low_rank"])
@pytest.mark.parametrize("k", [2, 70])
def test_sparse_transition_pairwise_routes(jn, module, route, k):
    n_src, n_dst = (7, 6) if k < 6 else (300, 120)
    src = _layer(jn, n_src, 4, 34)
    dst = _layer(jn, n_dst, 4, 35)
    make_route = (lambda: jn.DiagonalBilinearRoute(src_dim=4, dst_dim=4)) if route == "diagonal" else \
        (lambda: jn.LowRankBilinearRoute(src_dim=4, dst_dim=4, rank=3))
    rf = make_route().cuda()
    ref, nat = _pair(lambda **kw: jn.SparseTransition(route_fn=rf, topk=k, state_activation_fn=lambda x: x + 1.25,
                                                      val_proj_fn=_val_proj, state_proj_fn=_state_proj, **kw))
    # low-rank routes with k <= 64 take the reference's autograd route
    # (low_rank_pairwise_topk_forward_cuda, native_backend.py:5962-5993), the others the op
    with mock.patch.object(module, "transition_pairwise_topk", wraps=module.transition_pairwise_topk) as w, \
            mock.patch.object(module, "low_rank_pairwise_topk_forward_cuda",
                              wraps=module.low_rank_pairwise_topk_forward_cuda) as w_lr:
        got = nat.compute_delta(src, dst)
    assert w.call_count + w_lr.call_count > 0
    _close(ref.compute_delta(src, dst), got, atol=1e-5 if k < 6 else 1e-4, rtol=1e-5 if k < 6 else 1e-4)


def test_unsupported_scorer_kinds_raise_type_error(jn, module):
    """Kinds this backend does not implement raise TypeError -- the reference's "not here"
    signal (SparseTransition falls back on it, transition.py:620-623)."""
    layer = _layer(jn, 6, 4, 36)
    pw = jn.HadamardMLPPairwise(dim=4, hidden_dim=7).cuda()
    op = jn.Propagation(pairwise_fn=pw, implementation="native")
    with pytest.raises(TypeError):
        op.compute_delta(layer)


def test_transition_query_topk_native_entry(jn, module):
    """transition_query_topk has no Layer-API class; the reference reaches it through
    native_backend.transition_query_topk_native (native_backend.py:5857-5941). The
    expectation is the op's definition in torch: logits route(src, query)^T, top-k per query,
    softmax over the k, sender-weighted gather (jakal_net_native.cpp:7089-7246)."""
    import jakal_net.native_backend as nb

    g = torch.Generator(device="cuda").manual_seed(37)
    B, S, Q, D, k = 2, 300, 40, 16, 12
    src = torch.randn(B, S, D, device="cuda", generator=g)
    qv = torch.randn(B, Q, D, device="cuda", generator=g)
    sstate = torch.randn(B, S, device="cuda", generator=g)
    route = jn.LowRankBilinearRoute(src_dim=D, dst_dim=D, rank=8).cuda()
    sender = torch.nn.functional.softplus(sstate)
    with mock.patch.object(module, "transition_query_topk", wraps=module.transition_query_topk) as w:
        got = nb.transition_query_topk_native(route_fn=route, sender_strength=sender, src_val=src, query_val=qv,
                                              projected_state=sstate, projected_val=src, topk=k,
                                              query_block_size=16, source_block_size=128)
    assert w.call_count > 0
    with torch.no_grad():
        logits = route(src, qv).transpose(-1, -2)  # [B, Q, S]
        top = torch.topk(logits, k, dim=-1)
        wts = torch.softmax(top.values, dim=-1) * torch.gather(sender[:, None, :].expand(B, Q, S), -1, top.indices)
        exp_state = (wts * torch.gather(sstate[:, None, :].expand(B, Q, S), -1, top.indices)).sum(-1)
        gathered = torch.gather(src[:, None].expand(B, Q, S, D), 2, top.indices[..., None].expand(B, Q, k, D))
        exp_val = (wts[..., None] * gathered).sum(-2)
    assert torch.allclose(got.delta_state, exp_state, atol=1e-5, rtol=1e-5)
    assert torch.allclose(got.delta_val, exp_val, atol=1e-5, rtol=1e-5)


def _progressive_b(pb, implementation, prefix, dim, vocab, hidden, topk, window, expand, compress, layers=2):
    torch.manual_seed(3)
    specs = pb.build_progressive_b_stage_specs(prefix, lite_layers=layers, mid_layers=0, full_layers=0,
                                               lite_expand_ratio=expand / prefix,
                                               lite_compress_ratio=compress / prefix)
    return pb.ProgressiveBExampleLM(
        vocab_size=vocab, dim=dim, seq_nodes=prefix, stage_specs=specs, s_window=window, route_topk=topk,
        expanded_topk=topk, compressed_topk=topk, query_topk=topk, route_kind="low_rank_bilinear",
        pairwise_kind="low_rank_bilinear", route_hidden_dim=hidden, pairwise_hidden_dim=hidden,
        implementation=implementation).cuda().eval()


def _count_calls(module, fn):
    names = ("propagation_window", "propagation_topk", "transition_pairwise_topk", "propagation_dense",
             "transition_pairwise_dense", "propagation_query_dense", "transition_query_topk",
             "low_rank_pairwise_topk_forward_cuda")
    with contextlib.ExitStack() as stack:
        mocks = {n: stack.enter_context(mock.patch.object(module, n, wraps=getattr(module, n))) for n in names}
        out = fn()
    return out, {n: m.call_count for n, m in mocks.items() if m.call_count}



def test_progressive_b_query_block_f32(jn, module):
    """Config 4's architecture (low-rank scorers and routes, window S propagation, top-k B
    propagation, per-source transitions, query transition + causal query propagation) at a
    reduced size, f32: logits of the native run match the reference implementation."""
    pb = reference_shim.import_progressive_b()
    args = dict(prefix=128, dim=64, vocab=512, hidden=16, topk=8, window=32, expand=32, compress=16)
    ref = _progressive_b(pb, "reference", **args)
    nat = _progressive_b(pb, "native", **args)
    nat.load_state_dict(ref.state_dict())
    ids = torch.randint(0, 512, (2, 128), device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
    with torch.no_grad():
        want = ref.forward_query_block(ids, target_len=16)
        got, calls = _count_calls(module, lambda: nat.forward_query_block(ids, target_len=16))
    for op in ("propagation_window", "propagation_topk", "low_rank_pairwise_topk_forward_cuda"):
        assert calls.get(op, 0) > 0, calls
    rel = ((got - want).norm() / want.norm()).item()
    assert rel < 1e-4, rel


def test_progressive_b_query_block_bf16_autocast(jn, module):
    """The same model under bf16 autocast (config 4's precision): the native ops take bf16
    projections (the reference's at::matmul under autocast). The reference implementation
    rounds its scores to bf16 instead (modules.py:97), so the two runs pick different
    top-k members at near-ties; the logits agree to a few per cent."""
    pb = reference_shim.import_progressive_b()
    args = dict(prefix=256, dim=128, vocab=1024, hidden=64, topk=16, window=64, expand=64, compress=16)
    ref = _progressive_b(pb, "reference", **args)
    nat = _progressive_b(pb, "native", **args)
    nat.load_state_dict(ref.state_dict())
    ids = torch.randint(0, 1024, (2, 256), device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        want = ref.forward_query_block(ids, target_len=32).float()
        got, calls = _count_calls(module, lambda: nat.forward_query_block(ids, target_len=32).float())
    assert calls.get("propagation_window", 0) > 0 and calls.get("low_rank_pairwise_topk_forward_cuda", 0) > 0, calls
    assert torch.isfinite(got).all()
    rel = ((got - want).norm() / want.norm()).item()
    print(f"bf16 autocast logits: relative L2 difference native vs reference {rel:.3e}; calls {calls}")
    assert rel < 0.1, rel


@pytest.mark.parametrize("edge", ["softsign", "signed_abs"])
def test_config1_causal_dense_against_reference(jn, module, edge):
    """Config 1's shape and inputs (B2 N256 D128 R32 f32, causal window 255 = causal dense,
    val / state ~ N(0, 1), W ~ N(0, 1/sqrt(D)), w = ones, b = 0, seed 0) through the
    reference's SparsePropagation, native against reference."""
    torch.manual_seed(0)
    B, N, D, R = 2, 256, 128, 32
    g = torch.Generator().manual_seed(0)
    layer = jn.Layer(dim=D, num_nodes=N, state=torch.randn(B, N, generator=g).cuda(),
                     val=torch.randn(B, N, D, generator=g).cuda())
    pw = jn.LowRankBilinearPairwise(dim=D, rank=R)
    with torch.no_grad():
        pw.source_proj.weight.copy_(torch.randn(R, D, generator=g) / D ** 0.5)
        pw.target_proj.weight.copy_(torch.randn(R, D, generator=g) / D ** 0.5)
    pw = pw.cuda()
    kw = {} if edge == "softsign" else {"edge_compress_fn": signed_abs_softmax_edges}
    ref, nat = _pair(lambda **a: jn.SparsePropagation(pairwise_fn=pw, sparse_type="window", window=N - 1, **kw, **a))
    with mock.patch.object(module, "propagation_window", wraps=module.propagation_window) as w:
        got = nat.compute_delta(layer)
    assert w.call_count > 0
    _close(ref.compute_delta(layer), got, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("direction_only", [False, True])
def test_hierarchical_memory_level_write_and_propagation(jn, module, direction_only):
    """A causal-memory consumer (hierarchical_memory.py:35-136): one memory level's write
    (SparseTransition, signed-abs routes, softplus senders) from a sequence layer into the
    slots, then the slots' top-k propagation (signed-abs edges), native against reference,
    with every module entry point the level reaches wrapped."""
    from jakal_net.hierarchical_memory import _MemoryLevel

    def level(impl):
        torch.manual_seed(9)
        return _MemoryLevel(dim=32, num_slots=48, pairwise_kind="low_rank_bilinear", route_kind="low_rank_bilinear",
                            pairwise_rank=16, route_rank=16, pairwise_heads=1, route_heads=1,
                            pairwise_frozen_heads=0, route_frozen_heads=0, pairwise_anchor_heads=0,
                            route_anchor_heads=0, pairwise_anchor_kind="scaled_cosine",
                            route_anchor_kind="fixed_projection", memory_topk=6, memory_train_mode="topk",
                            memory_eval_mode="topk", eval_topk=None, implementation=impl,
                            direction_only_values=direction_only).cuda().eval()

    ref, nat = level("reference"), level("native")
    nat.load_state_dict(ref.state_dict())
    seq = _layer(jn, 200, 32, 90)
    names = ("propagation_topk", "transition_pairwise_topk", "low_rank_pairwise_topk_forward_cuda")
    with torch.no_grad():
        want_mem = ref.initialize(batch_size=2, device="cuda", dtype=torch.float32)
        want_w = ref.write.compute_delta(seq, want_mem)
        got_mem = nat.initialize(batch_size=2, device="cuda", dtype=torch.float32)
        with contextlib.ExitStack() as stack:
            mocks = {n: stack.enter_context(mock.patch.object(module, n, wraps=getattr(module, n))) for n in names}
            got_w = nat.write.compute_delta(seq, got_mem)
            mem = jn.Layer(dim=32, num_nodes=48, state=want_mem.state + want_w.delta_state,
                           val=want_mem.val + want_w.delta_val)
            got_p = nat.compute_propagation_delta(mem)
        want_p = ref.compute_propagation_delta(mem)
    assert mocks["propagation_topk"].call_count > 0, {n: m.call_count for n, m in mocks.items()}
    assert mocks["transition_pairwise_topk"].call_count + mocks["low_rank_pairwise_topk_forward_cuda"].call_count > 0
    _close(want_w, got_w, atol=1e-4, rtol=1e-4)
    _close(want_p, got_p, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("route", ["linear", "mlp", "full_bilinear"])
@pytest.mark.parametrize("k", [3, 0])
def test_node_and_full_bilinear_routes(jn, module, route, k):
    """Linear / MLP node routes (transition_dense, transition_topk) and the full-bilinear
    pairwise route, dense (k = 0) and sparse, native against reference."""
    src = _layer(jn, 40, 6, 60)
    dst = _layer(jn, 9, 6, 61)
    if route == "linear":
        make = lambda: jn.LinearRoute(src_dim=6, dst_nodes=9)  # noqa: E731
    elif route == "mlp":
        make = lambda: jn.MLPRoute(src_dim=6, dst_nodes=9, hidden_dim=11)  # noqa: E731
    else:
        make = lambda: jn.BilinearPairwiseRoute(src_dim=6, dst_dim=6, route_dim=5)  # noqa: E731
    rf = make().cuda()
    if k:
        ref, nat = _pair(lambda **kw: jn.SparseTransition(route_fn=rf, topk=k, state_activation_fn=lambda x: x + 1.25,
                                                          val_proj_fn=_val_proj, state_proj_fn=_state_proj, **kw))
        op = "transition_pairwise_topk" if route == "full_bilinear" else "transition_topk"
    else:
        ref, nat = _pair(lambda **kw: jn.Transition(route_fn=rf, state_activation_fn=lambda x: x + 1.25,
                                                    val_proj_fn=_val_proj, state_proj_fn=_state_proj, **kw))
        op = "transition_pairwise_dense" if route == "full_bilinear" else "transition_dense"
    with mock.patch.object(module, op, wraps=getattr(module, op)) as w:
        got = nat.compute_delta(src, dst)
    assert w.call_count > 0
    _close(ref.compute_delta(src, dst), got)
