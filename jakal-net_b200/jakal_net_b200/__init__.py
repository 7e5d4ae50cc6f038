"""B200-native (sm_100a) backend for the Jakal-Net operator hot path.

This module is a drop-in for the reference's native extension module: the reference
loader (``jakal_net.native_backend._load_native_module``, native_backend.py:98-160)
imports the module named by ``JAKAL_NET_NATIVE_MODULE``; with
``JAKAL_NET_NATIVE_MODULE=jakal_net_b200`` it reads ``supported_ops()``,
``supported_devices()`` and ``backend_name()`` from here and then calls the op functions
below positionally, exactly as it calls ``jakal_net_native`` (native_backend.py:5359-6021).

Every op runs on the GPU through ``libjakal_b200.so`` (C ABI in include/jakal_b200.h).
There is no CPU path: CPU tensors, unsupported kinds or dtypes raise instead of falling
back to another implementation.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from ._lib import JakalB200Error, check, load

__all__ = [
    "supported_ops",
    "supported_devices",
    "backend_name",
    "propagation_dense",
    "propagation_window",
    "propagation_query_dense",
    "propagation_topk",
    "propagation_window_topk",
    "masked_aggregate",
    "transition_query_topk",
    "transition_pairwise_topk",
    "lowrank_project",
    "lowrank_project_pair",
    "topk_aggregate",
    "JakalB200Error",
]

_LIBRARY = load()  # import fails loudly when the library is missing

_DTYPE_CODE = {torch.float32: _lib.JK_F32, torch.bfloat16: _lib.JK_BF16, torch.float16: _lib.JK_F16}
_EDGE_CODE = {
    "softsign": _lib.JK_SOFTSIGN,
    "signed_abs_softmax": _lib.JK_SIGNED_ABS_SOFTMAX,
    "signed_entmax15": _lib.JK_SIGNED_ENTMAX15,
}
_ROUTE_CODE = {
    "softmax": _lib.JK_SOFTMAX,
    "signed_abs_softmax": _lib.JK_SIGNED_ABS_SOFTMAX,
    "signed_entmax15": _lib.JK_SIGNED_ENTMAX15,
}
_MAX_K = 64
# MultiHeadPairwise aggregate -> jk_heads_t.combine (kernel_common.py:151-178 spec kinds
# multihead_{max,smoothmax,signed_smoothmax}_low_rank_bilinear)
_HEAD_COMBINE = {
    "max": _lib.JK_HEADS_MAX,
    "smoothmax": _lib.JK_HEADS_SMOOTHMAX,
    "signed_smoothmax": _lib.JK_HEADS_SIGNED_SMOOTHMAX,
}

_SUPPORTED_OPS = (
    "propagation_dense",
    "propagation_window",
    "propagation_query_dense",
    "propagation_topk",
    "transition_pairwise_dense",
    "transition_pairwise_topk",
    "transition_query_topk",
)


def supported_ops() -> list[str]:
    """Ops this module implements (jakal_net_native.cpp:5863-5912 contract). The
    ``*_cuda`` autograd entry points are deliberately not advertised: this backend is
    forward-only, and advertising them would route training through them
    (native_backend.py:659-667)."""
    return list(_SUPPORTED_OPS)


def supported_devices() -> list[str]:
    return ["cuda"]


def backend_name() -> str:
    return "b200_sm100a"


# ----------------------------------------------------------------------------- helpers
def _ptr(t: Optional[Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(name: str, t: Tensor) -> None:
    if not isinstance(t, Tensor):
        raise TypeError(f"{name} must be a tensor")
    if t.device.type != "cuda":
        raise RuntimeError(f"{name} must be a CUDA tensor in the b200_sm100a backend (got {t.device}).")


def _dtype_code(name: str, t: Tensor) -> int:
    code = _DTYPE_CODE.get(t.dtype)
    if code is None:
        raise RuntimeError(f"{name}: unsupported dtype {t.dtype}")
    return code


def _proj_dtype(val: Tensor, split3: bool = False) -> int:
    if split3:
        return _lib.JK_BF16X3
    if val.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError(
            "b200_sm100a scores low-rank projections on tcgen05 tensor cores; projections must be bf16 / f16, "
            f"or the three-plane split of f32 projections (got {val.dtype})."
        )
    return _DTYPE_CODE[val.dtype]


def _flatten_val(t: Tensor) -> Tensor:
    return t.reshape(-1, t.shape[-2], t.shape[-1]).contiguous()


def _flatten_state(t: Tensor) -> Tensor:
    return t.reshape(-1, t.shape[-1]).contiguous()


def lowrank_project(x: Tensor, weight: Tensor, core: Optional[Tensor] = None,
                    temperature: float = 1.0) -> Tensor:
    """round(x @ weight^T) [* core] [/ temperature] in x's dtype, padded to a multiple of
    64 columns (jakal_net_native.cpp:6236-6239, 6977-6986). x [..., D] -> [..., rp].

    f32 inputs (rank <= 32): the f32 projection (a plain f32 GEMM, like the reference's
    torch::matmul) is returned as three bf16 planes [h | m | l | 0] (rp = 128) whose six
    cross products the fused kernels sum -- an f32-accurate score (JK_BF16X3)."""
    _require_cuda("x", x)
    rank, dim = weight.shape
    if x.shape[-1] != dim:
        raise ValueError(f"projection weight expects dim {dim}, got {x.shape[-1]}")
    x2 = x.reshape(-1, dim).contiguous()
    if x.dtype == torch.float32:
        if rank > 32:
            raise RuntimeError(f"b200_sm100a f32 scoring supports score rank <= 32 (got {rank}).")
        proj = torch.matmul(x2, weight.detach().to(device=x.device, dtype=torch.float32).t())
        if core is not None:
            proj = proj * core.detach().reshape(-1).to(device=x.device, dtype=torch.float32)
        if float(temperature) != 1.0:
            proj = proj / float(temperature)
        proj = proj.contiguous()
        out = torch.empty((x2.shape[0], 128), device=x.device, dtype=torch.bfloat16)
        with torch.cuda.device(x.device):
            check(_LIBRARY.jk_split3_bf16(proj.data_ptr(), x2.shape[0], rank, out.data_ptr(), _stream(x.device)),
                  "jk_split3_bf16")
        return out.reshape(*x.shape[:-1], 128)
    code = _proj_dtype(x)
    w = weight.detach().to(device=x.device, dtype=x.dtype).contiguous()
    c = None if core is None else core.detach().reshape(-1).to(device=x.device, dtype=x.dtype).contiguous()
    rp = int(_LIBRARY.jk_padded_rank(rank))
    out = torch.empty((x2.shape[0], rp), device=x.device, dtype=x.dtype)
    with torch.cuda.device(x.device):
        check(
            _LIBRARY.jk_lowrank_project(x2.data_ptr(), x2.shape[0], dim, w.data_ptr(), rank, _ptr(c),
                                        float(temperature), code, out.data_ptr(), rp, _stream(x.device)),
            "jk_lowrank_project",
        )
    return out.reshape(*x.shape[:-1], rp)


def lowrank_project_pair(x: Tensor, weight: Tensor, weight2: Tensor, core: Optional[Tensor] = None,
                         temperature: float = 1.0) -> tuple[Tensor, Tensor]:
    """(lowrank_project(x, weight), lowrank_project(x, weight2, core, temperature)) in one
    pass over x (jk_lowrank_project_pair): bf16 / f16 x, rank <= 64; other cases take the
    two separate projections."""
    _require_cuda("x", x)
    rank, dim = weight.shape
    if (x.dtype == torch.float32 or rank > 64 or tuple(weight2.shape) != (rank, dim) or x.shape[-1] != dim):
        return lowrank_project(x, weight), lowrank_project(x, weight2, core=core, temperature=temperature)
    x2 = x.reshape(-1, dim).contiguous()
    w = weight.detach().to(device=x.device, dtype=x.dtype).contiguous()
    w2 = weight2.detach().to(device=x.device, dtype=x.dtype).contiguous()
    c = None if core is None else core.detach().reshape(-1).to(device=x.device, dtype=x.dtype).contiguous()
    out = torch.empty((x2.shape[0], 64), device=x.device, dtype=x.dtype)
    out2 = torch.empty((x2.shape[0], 64), device=x.device, dtype=x.dtype)
    with torch.cuda.device(x.device):
        check(
            _LIBRARY.jk_lowrank_project_pair(x2.data_ptr(), x2.shape[0], dim, w.data_ptr(), w2.data_ptr(), rank, _ptr(c),
                                             float(temperature), _proj_dtype(x), out.data_ptr(), out2.data_ptr(),
                                             _stream(x.device)),
            "jk_lowrank_project_pair",
        )
    return out.reshape(*x.shape[:-1], 64), out2.reshape(*x.shape[:-1], 64)


def _bias_tensor(bias: Optional[Tensor], device: torch.device, scale: float = 1.0) -> Optional[Tensor]:
    if bias is None:
        return None
    b = bias.detach().reshape(-1)
    if b.numel() == 0:
        return None
    if b.numel() != 1:
        raise RuntimeError("score bias must be a scalar")
    b = b.to(device=device, dtype=torch.float32)
    return b / scale if scale != 1.0 else b.contiguous()


class Heads:
    """Multi-head scorer of one call (jk_heads_t): the projection rows hold `heads` blocks of
    16 * kph columns; per-head scores plus `bias` [heads] are combined by `combine`."""

    def __init__(self, heads: int, kph: int, combine: int, bias: Optional[Tensor] = None):
        self.bias = bias  # keeps the device tensor alive for the call
        self.struct = _lib.JkHeads(int(heads), int(kph), int(combine), _ptr(bias))

    def ref(self):
        return ctypes.byref(self.struct)


def _multihead_project(x: Tensor, weight: Tensor, core: Optional[Tensor] = None, temperature: float = 1.0):
    """Per-head projections x @ weight[h]^T [* core[h]] [/ T] packed head-major into one
    projection row: head h at columns [16 kph h, 16 kph h + R), zeros elsewhere. weight
    [H, R, D], core [H, R]. Returns (proj [..., rp], kph)."""
    if x.dtype == torch.float32:
        raise RuntimeError("b200_sm100a multi-head scorers take bf16 / f16 inputs.")
    H, R, D = weight.shape
    rb = -(-R // 16) * 16
    if H * rb > 128:
        raise RuntimeError(f"b200_sm100a multi-head scorers need heads * roundup16(rank) <= 128 (got {H} x {R}).")
    w = weight.detach().new_zeros((H, rb, D))
    w[:, :R] = weight.detach()
    c = None
    if core is not None:
        c = core.detach().new_zeros((H, rb))
        c[:, :R] = core.detach().reshape(H, R)
        c = c.reshape(-1)
    return lowrank_project(x, w.reshape(H * rb, D), core=c, temperature=temperature), rb // 16


def _head_bias(bias: Optional[Tensor], heads: int, device: torch.device, scale: float = 1.0) -> Optional[Tensor]:
    if bias is None:
        return None
    b = bias.detach().reshape(-1).to(device=device, dtype=torch.float32)
    if b.numel() == 0:
        return None
    if b.numel() == 1:
        b = b.expand(heads)
    if b.numel() != heads:
        raise RuntimeError(f"multi-head bias must have {heads} entries (got {b.numel()}).")
    return (b / scale).contiguous()


def _diagonal_projections(target_val: Tensor, source_val: Tensor, w_hat: Tensor, temperature: float = 1.0):
    """Diagonal bilinear scorer (modules.py:37-53, 385-412): score = target . (source * w_hat).
    The projections are identity / diag(w_hat) GEMMs through jk_lowrank_project: one exact
    product per output, rounded once -- the reference's elementwise multiply."""
    D = target_val.shape[-1]
    if source_val.shape[-1] != D or w_hat.numel() != D:
        raise RuntimeError("diagonal bilinear scorer needs matching dims.")
    eye = torch.eye(D, device=target_val.device, dtype=torch.float32)
    row_proj = lowrank_project(target_val, eye)
    col_proj = lowrank_project(source_val, eye, core=w_hat, temperature=temperature)
    return row_proj, col_proj


def _pair_scorer(kind: str, weight: Tensor, bias, in_weight, in_bias, out_weight, out_bias, target_val: Tensor,
                 source_val: Tensor):
    """Projections of a pairwise spec (kernel_common.py:151-192): low_rank_bilinear,
    diagonal_bilinear (dim <= 128) or multihead_{max,smoothmax,signed_smoothmax}_low_rank_bilinear.
    Returns (row_proj [target], col_proj [source, * core], scalar bias tensor or None, Heads or None)."""
    if kind == "diagonal_bilinear":
        row_proj, col_proj = _diagonal_projections(target_val, source_val, weight)
        return row_proj, col_proj, _bias_tensor(bias, target_val.device), None
    if in_weight is None or out_weight is None:
        raise RuntimeError("Low-rank bilinear pairwise kernel is missing projection weights.")
    if in_bias is not None or out_bias is not None:
        raise RuntimeError("Low-rank bilinear projections take no bias.")
    if kind == "low_rank_bilinear":
        if target_val is source_val:  # propagation: both projections in one pass over the values
            row_proj, col_proj = lowrank_project_pair(target_val, out_weight, in_weight, core=weight)
        else:
            row_proj = lowrank_project(target_val, out_weight)                # target side
            col_proj = lowrank_project(source_val, in_weight, core=weight)    # source side, * w_hat
        return row_proj, col_proj, _bias_tensor(bias, target_val.device), None
    prefix, base = "multihead_", "_low_rank_bilinear"
    agg = kind[len(prefix):-len(base)] if kind.startswith(prefix) and kind.endswith(base) else None
    if agg not in _HEAD_COMBINE:
        raise RuntimeError(f"Unsupported pairwise kernel kind for b200_sm100a: {kind}")
    if in_weight.dim() != 3 or out_weight.dim() != 3:
        raise RuntimeError("multi-head projection weights must be [heads, rank, dim].")
    H = in_weight.shape[0]
    row_proj, kph = _multihead_project(target_val, out_weight)
    col_proj, _ = _multihead_project(source_val, in_weight, core=weight)
    heads = Heads(H, kph, _HEAD_COMBINE[agg], _head_bias(bias, H, target_val.device))
    return row_proj, col_proj, None, heads


def topk_aggregate(row_proj: Tensor, col_proj: Tensor, col_state: Tensor, col_val: Tensor, k: int, *,
                   window: int = -1, compress: int = _lib.JK_SOFTSIGN, col_sender: Optional[Tensor] = None,
                   bias: Optional[Tensor] = None, score_bias: float = 0.0,
                   out_dtype: Optional[torch.dtype] = None, return_selection: bool = False, split3: bool = False,
                   heads: Optional[Heads] = None, rows: Optional[tuple[int, int]] = None):
    """Raw fused top-k aggregate over already-projected inputs (jk_propagation_topk_forward,
    or jk_propagation_topk_forward_mh with a multi-head scorer).

    row_proj [B, T, rp], col_proj [B, S, rp], col_state [B, S], col_val [B, S, D].
    Returns (state [B, T], val [B, T, D]) and, with return_selection, also the selected
    scores (f32 [B, T, k]) and indices (int64 [B, T, k]).
    rows=(begin, count): compute only that row block (jk_propagation_topk_rows_forward;
    begin a multiple of 128); the other output rows are left unwritten (zeros here).
    """
    for name, t in (("row_proj", row_proj), ("col_proj", col_proj), ("col_state", col_state), ("col_val", col_val)):
        _require_cuda(name, t)
    B, T, rp = row_proj.shape
    S = col_proj.shape[1]
    D = col_val.shape[-1]
    dev = col_val.device
    out_dtype = out_dtype or col_val.dtype
    alloc = torch.empty if rows is None else torch.zeros
    out_state = alloc((B, T), device=dev, dtype=out_dtype)
    out_val = alloc((B, T, D), device=dev, dtype=out_dtype)
    scores = torch.empty((B, T, k), device=dev, dtype=torch.float32) if return_selection else None
    index = torch.empty((B, T, k), device=dev, dtype=torch.int64) if return_selection else None
    sender = None if col_sender is None else col_sender.to(col_state.dtype).contiguous()
    args = (row_proj.data_ptr(), col_proj.data_ptr(), B, T, S, rp, _proj_dtype(row_proj, split3),
            col_state.data_ptr(), _ptr(sender), _dtype_code("state", col_state),
            col_val.data_ptr(), D, _dtype_code("val", col_val),
            k, window, float(score_bias), _ptr(bias), compress,
            out_state.data_ptr(), out_val.data_ptr(), _dtype_code("out", out_state),
            _ptr(scores), _ptr(index))
    with torch.cuda.device(dev):
        if rows is not None:
            if heads is not None:
                raise RuntimeError("row blocks take the single-head scorer")
            check(_LIBRARY.jk_propagation_topk_rows_forward(*args[:4], int(rows[0]), int(rows[1]), *args[4:],
                                                            _stream(dev)),
                  "jk_propagation_topk_rows_forward")
        elif heads is None:
            check(_LIBRARY.jk_propagation_topk_forward(*args, _stream(dev)), "jk_propagation_topk_forward")
        else:
            check(_LIBRARY.jk_propagation_topk_forward_mh(*args, heads.ref(), _stream(dev)),
                  "jk_propagation_topk_forward_mh")
    if return_selection:
        return out_state, out_val, scores, index
    return out_state, out_val


def _propagation_topk_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name,
                           layer_val, projected_state, projected_val, topk: int, window: int):
    if edge_compress_name not in _EDGE_CODE:
        raise RuntimeError(
            "Only edge_compress_name in {softsign, signed_abs_softmax, signed_entmax15} is supported by the native backend."
        )
    if topk <= 0:
        raise RuntimeError("topk must be positive.")
    for name, t in (("layer_val", layer_val), ("projected_state", projected_state), ("projected_val", projected_val)):
        _require_cuda(name, t)
    batch_shape = layer_val.shape[:-2]
    n = layer_val.shape[-2]
    out_dim = projected_val.shape[-1]
    val = _flatten_val(layer_val)
    pstate = _flatten_state(projected_state)
    pval = _flatten_val(projected_val)
    k = min(int(topk), n)
    if k > _MAX_K:
        raise RuntimeError(f"b200_sm100a top-k supports k <= {_MAX_K} (got {k}).")
    row_proj, col_proj, bias_t, heads = _pair_scorer(kind, weight, bias, in_weight, in_bias, out_weight, out_bias,
                                                     val, val)
    same = projected_state.dtype == projected_val.dtype
    out_dtype = projected_val.dtype if same else torch.float32
    state, out = topk_aggregate(row_proj, col_proj, pstate, pval, k, window=window,
                                compress=_EDGE_CODE[edge_compress_name], bias=bias_t, out_dtype=out_dtype,
                                split3=val.dtype == torch.float32, heads=heads)
    state = state.to(projected_state.dtype).reshape(*batch_shape, n)
    out = out.to(projected_val.dtype).reshape(*batch_shape, n, out_dim)
    return state, out


def propagation_topk(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name,
                     layer_val, projected_state, projected_val, topk, target_block_size, source_block_size):
    """SparsePropagation(sparse_type="topk") forward: per target, top-k over every source
    (no causal mask), edges over the k, aggregate. Reference op: jakal_net_native.cpp:6305-6447
    (CUDA fast path :6355-6389). Block sizes are accepted for signature parity; the fused
    kernel tiles internally."""
    return _propagation_topk_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias,
                                  edge_compress_name, layer_val, projected_state, projected_val, topk, -1)


def propagation_window_topk(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name,
                            layer_val, projected_state, projected_val, window, topk, target_block_size=0,
                            source_block_size=0):
    """Window-intersect-top-k propagation: causal window mask (kernel_common.py:443-456),
    then top-k among the visible sources (rows with fewer visible sources use all of them),
    edges over the survivors (propagation.py:67-88). Not a reference op; the benchmark
    configurations that combine a causal window with top-k use it."""
    if window < 0:
        raise RuntimeError("window must be non-negative.")
    return _propagation_topk_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias,
                                  edge_compress_name, layer_val, projected_state, projected_val, topk, int(window))


def _route_projections(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                       hidden_weight, hidden_bias, out_weight, out_bias, temperature, src_val, dst_val):
    """Route projections (kernel_common.py:238-295): low_rank_bilinear_route,
    diagonal_bilinear_route (dim <= 128) or multihead_max_low_rank_bilinear_route;
    logits = (ps . pd + b) / T. Returns (src_proj / T, dst_proj, scalar bias / T or None,
    Heads or None)."""
    if route_kind not in ("low_rank_bilinear_route", "multihead_max_low_rank_bilinear_route",
                          "diagonal_bilinear_route"):
        raise TypeError(f"Unsupported pairwise route kind for b200_sm100a: {route_kind}")
    temperature = float(temperature)
    if temperature <= 0.0:
        raise RuntimeError("route temperature must be positive.")
    if route_kind == "diagonal_bilinear_route":
        if any(t is not None for t in (source_weight, source_bias, target_weight, target_bias, hidden_weight,
                                       hidden_bias, out_weight, out_bias)):
            raise TypeError("Diagonal routes take no projection / hidden layers.")
        dst_proj, src_proj = _diagonal_projections(dst_val, src_val, core_weight, temperature)
        return src_proj, dst_proj, _bias_tensor(bias, src_val.device, temperature), None
    if source_weight is None or target_weight is None:
        raise RuntimeError("Low-rank route kernel is missing projection weights.")
    if any(t is not None for t in (source_bias, target_bias, hidden_weight, hidden_bias, out_weight, out_bias)):
        raise TypeError("Low-rank route projections take no bias / hidden layers.")
    if route_kind == "multihead_max_low_rank_bilinear_route":
        # max_h(l_h) / T == max_h(l_h / T): every head's source projection and bias take the 1 / T
        H = source_weight.shape[0]
        src_proj, kph = _multihead_project(src_val, source_weight, core=core_weight, temperature=temperature)
        dst_proj, _ = _multihead_project(dst_val, target_weight)
        heads = Heads(H, kph, _lib.JK_HEADS_MAX, _head_bias(bias, H, src_val.device, temperature))
        return src_proj, dst_proj, None, heads
    src_proj = lowrank_project(src_val, source_weight, core=core_weight, temperature=temperature)
    dst_proj = lowrank_project(dst_val, target_weight)
    return src_proj, dst_proj, _bias_tensor(bias, src_val.device, temperature), None


def transition_query_topk(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                          hidden_weight, hidden_bias, out_weight, out_bias, temperature, sender_strength, src_val,
                          query_val, projected_state, projected_val, topk, query_block_size, source_block_size,
                          use_cuda_reduce=True):
    """Per-query transition (jakal_net_native.cpp:7089-7246): each query slot takes its
    top-k sources by route logit, softmax over the k, sender-weighted gather."""
    for name, t in (("sender_strength", sender_strength), ("src_val", src_val), ("query_val", query_val),
                    ("projected_state", projected_state), ("projected_val", projected_val)):
        _require_cuda(name, t)
    if topk <= 0:
        raise RuntimeError("topk must be positive.")
    batch_shape = query_val.shape[:-2]
    n_query = query_val.shape[-2]
    n_src = src_val.shape[-2]
    out_dim = projected_val.shape[-1]
    sv = _flatten_val(src_val)
    qv = _flatten_val(query_val)
    k = min(int(topk), n_src)
    if k > _MAX_K:
        raise RuntimeError(f"b200_sm100a top-k supports k <= {_MAX_K} (got {k}).")
    src_proj, q_proj, bias_t, heads = _route_projections(route_kind, source_weight, source_bias, target_weight,
                                                         target_bias, core_weight, bias, hidden_weight, hidden_bias,
                                                         out_weight, out_bias, temperature, sv, qv)
    pstate = _flatten_state(projected_state)
    sender = _flatten_state(sender_strength).to(pstate.dtype)
    pval = _flatten_val(projected_val)
    same = projected_state.dtype == projected_val.dtype
    out_dtype = projected_val.dtype if same else torch.float32
    state, out = topk_aggregate(q_proj, src_proj, pstate, pval, k, window=-1, compress=_lib.JK_SOFTMAX,
                                col_sender=sender, bias=bias_t, out_dtype=out_dtype, split3=sv.dtype == torch.float32,
                                heads=heads)
    return (state.to(projected_state.dtype).reshape(*batch_shape, n_query),
            out.to(projected_val.dtype).reshape(*batch_shape, n_query, out_dim))


def transition_pairwise_topk(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                             hidden_weight, hidden_bias, out_weight, out_bias, temperature, sender_strength, src_val,
                             dst_val, projected_state, projected_val, topk, src_block_size, dst_block_size,
                             route_compress_name="softmax"):
    """SparseTransition forward (jakal_net_native.cpp:6916-7087): each source takes its
    top-k destinations by route logit, routes compressed over the k, sender-weighted
    scatter-add into the destinations."""
    for name, t in (("sender_strength", sender_strength), ("src_val", src_val), ("dst_val", dst_val),
                    ("projected_state", projected_state), ("projected_val", projected_val)):
        _require_cuda(name, t)
    if topk <= 0:
        raise RuntimeError("topk must be positive.")
    if route_compress_name not in _ROUTE_CODE:
        raise RuntimeError(f"Unsupported route compress {route_compress_name!r}")
    batch_shape = src_val.shape[:-2]
    n_src = src_val.shape[-2]
    n_dst = dst_val.shape[-2]
    out_dim = projected_val.shape[-1]
    sv = _flatten_val(src_val)
    dv = _flatten_val(dst_val)
    k = min(int(topk), n_dst)
    if k > _MAX_K:
        raise RuntimeError(f"b200_sm100a top-k supports k <= {_MAX_K} (got {k}).")
    src_proj, dst_proj, bias_t, heads = _route_projections(route_kind, source_weight, source_bias, target_weight,
                                                           target_bias, core_weight, bias, hidden_weight,
                                                           hidden_bias, out_weight, out_bias, temperature, sv, dv)
    pstate = _flatten_state(projected_state)
    sender = _flatten_state(sender_strength).to(pstate.dtype)
    pval = _flatten_val(projected_val)
    B = sv.shape[0]
    dev = sv.device
    same = projected_state.dtype == projected_val.dtype
    out_dtype = projected_val.dtype if same else torch.float32
    accum = torch.empty(B * n_dst * (out_dim + 1) + 4, device=dev, dtype=torch.float32)
    out_state = torch.empty((B, n_dst), device=dev, dtype=out_dtype)
    out_val = torch.empty((B, n_dst, out_dim), device=dev, dtype=out_dtype)
    args = (src_proj.data_ptr(), dst_proj.data_ptr(), B, n_src, n_dst, src_proj.shape[-1],
            _proj_dtype(src_proj, sv.dtype == torch.float32),
            pstate.data_ptr(), sender.data_ptr(), _dtype_code("state", pstate),
            pval.data_ptr(), out_dim, _dtype_code("val", pval),
            k, 0.0, _ptr(bias_t), _ROUTE_CODE[route_compress_name], accum.data_ptr(),
            out_state.data_ptr(), out_val.data_ptr(), _dtype_code("out", out_state))
    with torch.cuda.device(dev):
        if heads is None:
            check(_LIBRARY.jk_transition_pairwise_topk_forward(*args, _stream(dev)),
                  "jk_transition_pairwise_topk_forward")
        else:
            check(_LIBRARY.jk_transition_pairwise_topk_forward_mh(*args, heads.ref(), _stream(dev)),
                  "jk_transition_pairwise_topk_forward_mh")
    return (out_state.to(projected_state.dtype).reshape(*batch_shape, n_dst),
            out_val.to(projected_val.dtype).reshape(*batch_shape, n_dst, out_dim))


def _value_planes(pval: Tensor, proj_dtype: torch.dtype):
    """Values for the window-kernel value GEMM: padded to 64 columns; f32 values become bf16
    hi + lo planes (both multiplied by the hi + lo edge planes). Returns (val, val_lo, pad)."""
    out_dim = pval.shape[-1]
    pad = (-out_dim) % 64
    if pad:
        pval = torch.nn.functional.pad(pval, (0, pad))
    pval_lo = None
    if proj_dtype == torch.float32:
        pval = pval.float().contiguous()
        hi = torch.empty(pval.shape, device=pval.device, dtype=torch.bfloat16)
        pval_lo = torch.empty_like(hi)
        with torch.cuda.device(pval.device):
            check(_LIBRARY.jk_split2_bf16(pval.data_ptr(), pval.numel(), hi.data_ptr(), pval_lo.data_ptr(),
                                          _stream(pval.device)), "jk_split2_bf16")
        pval = hi
    elif pval.dtype != proj_dtype:
        pval = pval.to(proj_dtype)
    return pval.contiguous(), pval_lo, pad


def transition_pairwise_dense(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                              hidden_weight, hidden_bias, out_weight, out_bias, route_compress_name, temperature,
                              sender_strength, src_val, dst_val, projected_state, projected_val, src_block_size,
                              dst_block_size):
    """Dense pairwise Transition forward (jakal_net_native.cpp:6705-6914; transition.py:238-254):
    routes of every source compressed over all destinations, sender-weighted, accumulated into
    the destinations. Two fused launches: per-source route statistics, then the per-destination
    aggregate with per-column normalisation."""
    for name, t in (("sender_strength", sender_strength), ("src_val", src_val), ("dst_val", dst_val),
                    ("projected_state", projected_state), ("projected_val", projected_val)):
        _require_cuda(name, t)
    if route_compress_name not in _ROUTE_CODE:
        raise RuntimeError(f"Unsupported route compress {route_compress_name!r}")
    batch_shape = src_val.shape[:-2]
    n_src = src_val.shape[-2]
    n_dst = dst_val.shape[-2]
    out_dim = projected_val.shape[-1]
    sv = _flatten_val(src_val)
    dv = _flatten_val(dst_val)
    src_proj, dst_proj, bias_t, heads = _route_projections(route_kind, source_weight, source_bias, target_weight,
                                                           target_bias, core_weight, bias, hidden_weight,
                                                           hidden_bias, out_weight, out_bias, temperature, sv, dv)
    pstate = _flatten_state(projected_state)
    sender = _flatten_state(sender_strength).to(pstate.dtype).contiguous()
    pval, pval_lo, pad = _value_planes(_flatten_val(projected_val), sv.dtype)
    B = sv.shape[0]
    dev = sv.device
    same = projected_state.dtype == projected_val.dtype
    out_dtype = projected_val.dtype if same else torch.float32
    stats = torch.empty(B * n_src * 3, device=dev, dtype=torch.float32)
    out_state = torch.empty((B, n_dst), device=dev, dtype=out_dtype)
    out_val = torch.empty((B, n_dst, pval.shape[-1]), device=dev, dtype=out_dtype)
    args = (src_proj.data_ptr(), dst_proj.data_ptr(), B, n_src, n_dst, src_proj.shape[-1],
            _proj_dtype(src_proj, sv.dtype == torch.float32),
            pstate.data_ptr(), sender.data_ptr(), _dtype_code("state", pstate),
            pval.data_ptr(), _ptr(pval_lo), pval.shape[-1],
            0.0, _ptr(bias_t), _ROUTE_CODE[route_compress_name], stats.data_ptr(),
            out_state.data_ptr(), out_val.data_ptr(), _dtype_code("out", out_state))
    with torch.cuda.device(dev):
        if heads is None:
            check(_LIBRARY.jk_transition_pairwise_dense_forward(*args, _stream(dev)),
                  "jk_transition_pairwise_dense_forward")
        else:
            check(_LIBRARY.jk_transition_pairwise_dense_forward_mh(*args, heads.ref(), _stream(dev)),
                  "jk_transition_pairwise_dense_forward_mh")
    if pad:
        out_val = out_val[..., :out_dim]
    return (out_state.to(projected_state.dtype).reshape(*batch_shape, n_dst),
            out_val.to(projected_val.dtype).reshape(*batch_shape, n_dst, out_dim))


def masked_aggregate(row_proj: Tensor, col_proj: Tensor, col_state: Tensor, col_val: Tensor, *, window: int = -1,
                     compress: int = _lib.JK_SOFTSIGN, bias: Optional[Tensor] = None, score_bias: float = 0.0,
                     out_dtype: Optional[torch.dtype] = None, split3: bool = False,
                     col_val_lo: Optional[Tensor] = None, heads: Optional[Heads] = None):
    """Raw fused window / dense aggregate over already-projected inputs
    (jk_propagation_window_forward). row_proj [B, T, rp], col_proj [B, S, rp], col_state [B, S],
    col_val [B, S, D] in the projections' dtype, D a multiple of 64. window -1 = dense."""
    for name, t in (("row_proj", row_proj), ("col_proj", col_proj), ("col_state", col_state), ("col_val", col_val)):
        _require_cuda(name, t)
    B, T, rp = row_proj.shape
    S = col_proj.shape[1]
    D = col_val.shape[-1]
    dev = col_val.device
    out_dtype = out_dtype or col_val.dtype
    out_state = torch.empty((B, T), device=dev, dtype=out_dtype)
    out_val = torch.empty((B, T, D), device=dev, dtype=out_dtype)
    args = (row_proj.data_ptr(), col_proj.data_ptr(), B, T, S, rp, _proj_dtype(row_proj, split3),
            col_state.data_ptr(), _dtype_code("state", col_state), col_val.data_ptr(), _ptr(col_val_lo), D,
            int(window), float(score_bias), _ptr(bias), compress,
            out_state.data_ptr(), out_val.data_ptr(), _dtype_code("out", out_state))
    with torch.cuda.device(dev):
        if heads is None:
            check(_LIBRARY.jk_propagation_window_forward(*args, _stream(dev)), "jk_propagation_window_forward")
        else:
            check(_LIBRARY.jk_propagation_window_forward_mh(*args, heads.ref(), _stream(dev)),
                  "jk_propagation_window_forward_mh")
    return out_state, out_val


def _masked_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, target_val,
                 source_val, projected_state, projected_val, window: int, source_state=None):
    if edge_compress_name not in _EDGE_CODE:
        raise RuntimeError(
            "Only edge_compress_name in {softsign, signed_abs_softmax, signed_entmax15} is supported by the native backend."
        )
    for name, t in (("target_val", target_val), ("source_val", source_val), ("projected_state", projected_state),
                    ("projected_val", projected_val)):
        _require_cuda(name, t)
    batch_shape = target_val.shape[:-2]
    n_t = target_val.shape[-2]
    out_dim = projected_val.shape[-1]
    tv = _flatten_val(target_val)
    sv = _flatten_val(source_val)
    pstate = _flatten_state(projected_state)
    pval = _flatten_val(projected_val)
    if source_state is not None and source_state.numel() != 0:
        # edges weighted by the source state (jakal_net_native.cpp:6010-6013) == folding the
        # weight into the aggregated inputs
        ss = _flatten_state(source_state).float()
        pstate = (pstate.float() * ss).to(pstate.dtype)
        pval = (pval.float() * ss[..., None]).to(pval.dtype)
    f32 = tv.dtype == torch.float32
    pval, pval_lo, pad = _value_planes(pval, tv.dtype)
    row_proj, col_proj, bias_t, heads = _pair_scorer(kind, weight, bias, in_weight, in_bias, out_weight, out_bias,
                                                     tv, sv)
    same = projected_state.dtype == projected_val.dtype
    out_dtype = projected_val.dtype if same else torch.float32
    st, out = masked_aggregate(row_proj, col_proj, pstate, pval, window=window,
                               compress=_EDGE_CODE[edge_compress_name], bias=bias_t,
                               out_dtype=out_dtype, split3=f32, col_val_lo=pval_lo, heads=heads)
    if pad:
        out = out[..., :out_dim]
    return (st.to(projected_state.dtype).reshape(*batch_shape, n_t),
            out.to(projected_val.dtype).reshape(*batch_shape, n_t, out_dim))


def propagation_window(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, layer_val,
                       projected_state, projected_val, window, target_block_size, source_block_size):
    """SparsePropagation(sparse_type="window") forward: causal window [t - window, t], edges
    compressed over the visible sources, aggregate (jakal_net_native.cpp:6190-6303;
    propagation.py:453-480)."""
    if window < 0:
        raise RuntimeError("window must be non-negative.")
    return _masked_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, layer_val,
                        layer_val, projected_state, projected_val, int(window))


def propagation_dense(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, layer_val,
                      projected_state, projected_val, source_state, target_block_size, source_block_size):
    """Dense Propagation forward: every (target, source) pair (jakal_net_native.cpp:5962-6076;
    propagation.py:207-220)."""
    return _masked_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, layer_val,
                        layer_val, projected_state, projected_val, -1, source_state)


def propagation_query_dense(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name,
                            query_val, source_val, projected_state, projected_val, query_block_size,
                            source_block_size):
    """Dense query propagation: query rows score every source row (jakal_net_native.cpp:6078-6188)."""
    return _masked_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, query_val,
                        source_val, projected_state, projected_val, -1)
