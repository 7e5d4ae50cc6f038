"""B200-native (sm_100a) backend for the Jakal-Net operator hot path.

This module is a drop-in for the reference's native extension module: the reference
loader (``jakal_net.native_backend._load_native_module``, native_backend.py:98-160)
imports the module named by ``JAKAL_NET_NATIVE_MODULE``; with
``JAKAL_NET_NATIVE_MODULE=jakal_net_b200`` it reads ``supported_ops()``,
``supported_devices()`` and ``backend_name()`` from here and then calls the op functions
below positionally, exactly as it calls ``jakal_net_native`` (native_backend.py:5359-6021).

Every op runs on the GPU through ``libjakal_b200.so`` (C ABI in include/jakal_b200.h).
There is no CPU path: CPU tensors and unsupported compressors raise ``RuntimeError``;
scorer / route kinds this backend does not implement raise ``TypeError`` (the error the
reference's own dispatch treats as "not supported here", transition.py:620-623).

Two kernel families serve every op:
  * the fused kernels (tcgen05 score tiles kept on chip, streaming top-k, aggregate) for
    k <= 64 and single-head scorers of padded rank <= 128 with 16-bit projections, or f32
    projections of rank <= 32 (three-plane split), and multi-head scorers within the kernel
    head limits;
  * the select-aggregate kernel (jk_select_aggregate_forward) over materialised f32 score
    blocks -- a plain GEMM of the projections -- for everything else the reference accepts:
    any k, any score rank, f32 projections of any rank, diagonal / full bilinear scorers of
    any width. It is exact (radix select) and reproduces the reference's blocked paths that
    take any k (jakal_net_native.cpp:6390-6447, 6916-7087, 7089-7246).
Under CUDA autocast the scorer inputs are cast to the autocast dtype before the projection
GEMMs, as the reference's at::matmul inside its extension is (jakal_net_native.cpp:6236-6239
runs within the caller's autocast region), and the aggregated values / states are cast to it
as autocast casts the reference's own einsum / bmm aggregates; accumulation is f32 and the
outputs keep the dtypes of the projected inputs.
"""
from __future__ import annotations

import contextlib
import ctypes
import functools
import threading
import weakref
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
_MAX_K = 64  # fused kernels; larger k takes the select-aggregate kernel
# f32 score elements per materialised block of the select-aggregate path (256 MiB)
_SCORE_BUDGET = 1 << 26
_TLS = threading.local()
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
    "transition_dense",
    "transition_topk",
    # training: the per-source sparse transition's autograd route (native_backend.py:5962-5975)
    "low_rank_pairwise_topk_forward_cuda",
    "low_rank_pairwise_topk_backward_cuda",
    "query_topk_reduce_backward_cuda",
    "softsign_backward_cuda",
    "softmax_backward_cuda",
    # the propagation autograd routes (behind the reference's experimental-training switch,
    # native_backend.py:5512-5565, 5600-5612)
    "low_rank_propagation_topk_forward_cuda",
    "low_rank_propagation_window_forward_cuda",
    "low_rank_propagation_window_signed_abs_forward_cuda",
    "low_rank_propagation_causal_dense_signed_abs_forward_cuda",
)


def supported_ops() -> list[str]:
    """Ops this module implements (jakal_net_native.cpp:5863-5912 contract), including the
    CUDA entry points of the autograd routes: the per-source sparse transition's
    (native_backend.py:659-667, 4408-4601, 5962-5975) and the top-k / window propagation's
    (:4815-4966, 5143-5357; the reference takes those only under its experimental-training
    switch). The signed_entmax15 routes also need the reference's torch.ops.jakal_net
    entmax ops, so they stay on the reference."""
    return list(_SUPPORTED_OPS)


def supported_devices() -> list[str]:
    return ["cuda"]


def backend_name() -> str:
    return "b200_sm100a"


# ----------------------------------------------------------------------------- helpers
def _entry(fn):
    """Op entry: records the caller's CUDA autocast dtype (the scorer inputs follow it, see
    the module docstring), then runs the op with autocast and autograd off -- the module's
    own torch calls are plain library work on already-decided dtypes, and its outputs are
    fresh tensors like the reference extension's (no autograd graph)."""

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        # plain flag toggles (not the context managers): an op is called per layer of a model
        # step, and the host time of every call adds to the step when the GPU waits on it
        prev = getattr(_TLS, "autocast", None)
        prev_casts = getattr(_TLS, "casts", None)
        _TLS.casts = {}
        ac_on = torch.is_autocast_enabled("cuda")
        grad_on = torch.is_grad_enabled()
        _TLS.autocast = torch.get_autocast_dtype("cuda") if ac_on else None
        if ac_on:
            torch.set_autocast_enabled("cuda", False)
        if grad_on:
            torch.set_grad_enabled(False)
        try:
            return fn(*args, **kwargs)
        finally:
            if grad_on:
                torch.set_grad_enabled(True)
            if ac_on:
                torch.set_autocast_enabled("cuda", True)
            _TLS.autocast = prev
            _TLS.casts = prev_casts

    return wrapper


def _autocast_cast(x: Tensor, ac: torch.dtype) -> Tensor:
    """x.to(ac), computed once per op call for one tensor (an op often scores and aggregates
    the same layer values, and reshaped views of it share the key)."""
    casts = getattr(_TLS, "casts", None)
    if casts is None:
        return x.to(ac)
    key = (x.data_ptr(), tuple(x.shape), tuple(x.stride()), ac)
    hit = casts.get(key)
    if hit is None:
        hit = casts[key] = x.to(ac)
    return hit


def _scorer_input(x: Tensor) -> Tensor:
    """The scorer (projection GEMM) input in the dtype the reference's at::matmul would use:
    f32 inputs are cast to the caller's autocast dtype when an op was called under CUDA
    autocast."""
    ac = getattr(_TLS, "autocast", None)
    if ac is not None and x.dtype == torch.float32:
        return _autocast_cast(x, ac)
    return x


def _aggregate_input(x: Tensor) -> Tensor:
    """An aggregated operand (projected state / value, sender strength) in the dtype the
    caller's autocast gives the reference's own aggregate: under CUDA autocast its einsum /
    bmm aggregates (propagation.py:215-219, transition.py:246-254) run in the autocast dtype,
    so f32 operands are cast to it; accumulation stays f32 and the outputs keep the dtype of
    the projected inputs."""
    ac = getattr(_TLS, "autocast", None)
    if ac is not None and x.dtype == torch.float32:
        return _autocast_cast(x, ac)
    return x


@contextlib.contextmanager
def _exact_f32_matmul():
    """f32 GEMMs in full f32 (TF32 off) for the duration of the block: the projections and
    score blocks of f32 inputs follow the reference's f32 torch::matmul."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _ptr(t: Optional[Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    """The raw handle of the current torch stream of `device`."""
    return torch._C._cuda_getCurrentRawStream(device.index if device.index is not None else torch.cuda.current_device())


def _on(device: torch.device):
    """Makes `device` current for the block (no guard when it already is)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


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


_PARAM_CASTS: dict = {}


def _cast_param(w: Tensor, device: torch.device, dtype: torch.dtype) -> Tensor:
    """w (a weight the caller owns, e.g. a module parameter) detached, on `device` in `dtype`,
    contiguous. Casts are kept per tensor object and reused while its version counter is
    unchanged (every in-place update, such as an optimizer step, bumps it), so a model's
    f32 weights are not cast again on every call."""
    if w.dtype == dtype and w.device == device:
        return w.detach().contiguous()
    key = (id(w), dtype, device)
    hit = _PARAM_CASTS.get(key)
    if hit is not None and hit[0]() is w and hit[1] == w._version:
        return hit[2]
    out = w.detach().to(device=device, dtype=dtype).contiguous()
    if len(_PARAM_CASTS) > 1024:
        _PARAM_CASTS.clear()
    _PARAM_CASTS[key] = (weakref.ref(w), w._version, out)
    return out


def _pad_dim8(x2: Tensor, w: Tensor) -> tuple[Tensor, Tensor]:
    """Zero-pads the contraction dim of a projection to a multiple of 8 (16-byte TMA rows);
    the padded columns add exact zeros to every dot product."""
    pad = (-x2.shape[-1]) % 8
    if pad:
        x2 = torch.nn.functional.pad(x2, (0, pad))
        w = torch.nn.functional.pad(w, (0, pad))
    return x2.contiguous(), w.contiguous()


def lowrank_project(x: Tensor, weight: Tensor, core: Optional[Tensor] = None,
                    temperature: float = 1.0) -> Tensor:
    """round(x @ weight^T) [* core] [/ temperature] in x's dtype, padded to a multiple of
    64 columns (jakal_net_native.cpp:6236-6239, 6977-6986). x [..., D] -> [..., rp].
    16-bit x: rank <= 128, any D (zero-padded to a multiple of 8).

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
            raise RuntimeError(f"b200_sm100a three-plane f32 scoring supports score rank <= 32 (got {rank}).")
        proj = _generic_project(x2, weight, core, temperature)
        out = torch.empty((x2.shape[0], 128), device=x.device, dtype=torch.bfloat16)
        with _on(x.device):
            check(_LIBRARY.jk_split3_bf16(proj.data_ptr(), x2.shape[0], rank, out.data_ptr(), _stream(x.device)),
                  "jk_split3_bf16")
        return out.reshape(*x.shape[:-1], 128)
    code = _proj_dtype(x)
    if rank > 128:
        raise RuntimeError(f"b200_sm100a fused projections support score rank <= 128 (got {rank}).")
    x2, w = _pad_dim8(x2, _cast_param(weight, x.device, x.dtype))
    c = None if core is None else _cast_param(core, x.device, x.dtype).reshape(-1)
    rp = int(_LIBRARY.jk_padded_rank(rank))
    out = torch.empty((x2.shape[0], rp), device=x.device, dtype=x.dtype)
    with _on(x.device):
        check(
            _LIBRARY.jk_lowrank_project(x2.data_ptr(), x2.shape[0], x2.shape[1], w.data_ptr(), rank, _ptr(c),
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
    x2, w = _pad_dim8(x.reshape(-1, dim), _cast_param(weight, x.device, x.dtype))
    _, w2 = _pad_dim8(x2[:0, :dim], _cast_param(weight2, x.device, x.dtype))
    c = None if core is None else _cast_param(core, x.device, x.dtype).reshape(-1)
    out = torch.empty((x2.shape[0], 64), device=x.device, dtype=x.dtype)
    out2 = torch.empty((x2.shape[0], 64), device=x.device, dtype=x.dtype)
    with _on(x.device):
        check(
            _LIBRARY.jk_lowrank_project_pair(x2.data_ptr(), x2.shape[0], x2.shape[1], w.data_ptr(), w2.data_ptr(),
                                             rank, _ptr(c), float(temperature), _proj_dtype(x), out.data_ptr(),
                                             out2.data_ptr(), _stream(x.device)),
            "jk_lowrank_project_pair",
        )
    return out.reshape(*x.shape[:-1], 64), out2.reshape(*x.shape[:-1], 64)


def _generic_project(x2: Tensor, weight: Optional[Tensor], core: Optional[Tensor] = None,
                     temperature: float = 1.0) -> Tensor:
    """Projection for the select-aggregate path, with the reference's rounding points
    (jakal_net_native.cpp:6236-6239, 6977-6986): p = x @ weight^T (weight None: the
    identity), then * core, then / temperature, each in x's dtype; returned as f32."""
    with _exact_f32_matmul():
        p = x2 if weight is None else torch.matmul(x2, weight.detach().to(device=x2.device, dtype=x2.dtype).t())
    if core is not None:
        p = p * core.detach().reshape(-1).to(device=x2.device, dtype=x2.dtype)
    if float(temperature) != 1.0:
        p = p / float(temperature)
    return p.float().contiguous()


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
        raise TypeError("b200_sm100a multi-head scorers take bf16 / f16 inputs.")
    H, R, D = weight.shape
    rb = -(-R // 16) * 16
    if H * rb > 128:
        raise TypeError(f"b200_sm100a multi-head scorers need heads * roundup16(rank) <= 128 (got {H} x {R}).")
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


# ----------------------------------------------------------------------------- scorers
class Scorer:
    """Projections of one call. fused: 16-bit (or three-plane f32) padded projections for
    the fused kernels, with `heads` for multi-head scorers; otherwise f32 projections
    [B, rows, R] for the select-aggregate path. `bias` is the scalar device bias or None."""

    def __init__(self, row: Tensor, col: Tensor, bias: Optional[Tensor], fused: bool,
                 heads: Optional[Heads] = None, split3: bool = False):
        self.row, self.col, self.bias, self.fused, self.heads, self.split3 = row, col, bias, fused, heads, split3


def _fused_rank_ok(x: Tensor, rank: int) -> bool:
    if x.dtype == torch.float32:
        return rank <= 32
    return x.dtype in (torch.bfloat16, torch.float16) and rank <= 128


def _single_scorer(tx: Tensor, sx: Tensor, t_weight: Optional[Tensor], s_weight: Optional[Tensor],
                   core: Optional[Tensor], temperature: float, bias: Optional[Tensor], rank: int,
                   fused: bool, pair: bool = False) -> Scorer:
    """Single-head low-rank form shared by every single-head kind: row = tx @ t_weight^T,
    col = (sx @ s_weight^T) * core / temperature (a weight of None is the identity).

    f32 inputs whose whole score matrix fits one materialised block take the
    select-aggregate path even when the fused three-plane form would apply: it scores,
    compresses and aggregates in plain f32 like the reference's f32 kernels."""
    pairs = (tx.numel() // max(1, tx.shape[-1])) * sx.shape[-2]
    if tx.dtype == torch.float32 and pairs <= _SCORE_BUDGET:
        fused = False
    if fused and _fused_rank_ok(tx, rank):
        dim = tx.shape[-1]
        eye = None
        if t_weight is None or s_weight is None:
            eye = torch.eye(dim, device=tx.device, dtype=torch.float32)
        tw = eye if t_weight is None else t_weight
        sw = eye if s_weight is None else s_weight
        if pair and tw.shape == sw.shape:
            row, col = lowrank_project_pair(tx, tw, sw, core=core, temperature=temperature)
        else:
            row = lowrank_project(tx, tw)
            col = lowrank_project(sx, sw, core=core, temperature=temperature)
        return Scorer(row, col, bias, True, split3=tx.dtype == torch.float32)
    row = _generic_project(tx.reshape(-1, tx.shape[-1]), t_weight).reshape(*tx.shape[:-1], -1)
    col = _generic_project(sx.reshape(-1, sx.shape[-1]), s_weight, core, temperature).reshape(*sx.shape[:-1], -1)
    return Scorer(row, col, bias, False)


def _pair_scorer(kind: str, weight: Tensor, bias, in_weight, in_bias, out_weight, out_bias, target_val: Tensor,
                 source_val: Tensor, fused: bool = True) -> Scorer:
    """Projections of a pairwise spec (kernel_common.py:151-212): low_rank_bilinear,
    diagonal_bilinear, bilinear (full D x D: score = t . (W s), modules.py:56-72) or
    multihead_{max,smoothmax,signed_smoothmax}_low_rank_bilinear. `fused` False forces the
    select-aggregate form (e.g. k > 64). Other kinds raise TypeError."""
    tx, sx = _scorer_input(target_val), _scorer_input(source_val)
    if tx.dtype != sx.dtype:
        raise RuntimeError("target and source values must share a dtype.")
    dev = target_val.device
    if kind == "diagonal_bilinear":
        dim = tx.shape[-1]
        if weight is None or weight.numel() != dim:
            raise RuntimeError("diagonal bilinear scorer needs a weight of the value dim.")
        return _single_scorer(tx, sx, None, None, weight, 1.0, _bias_tensor(bias, dev), dim, fused)
    if kind == "bilinear":
        dim = tx.shape[-1]
        if weight is None or tuple(weight.shape) != (dim, dim):
            raise RuntimeError("bilinear scorer needs a [dim, dim] weight.")
        return _single_scorer(tx, sx, None, weight, None, 1.0, _bias_tensor(bias, dev), dim, fused)
    if kind == "low_rank_bilinear":
        if in_weight is None or out_weight is None:
            raise RuntimeError("Low-rank bilinear pairwise kernel is missing projection weights.")
        if in_bias is not None or out_bias is not None:
            raise TypeError("Low-rank bilinear projections take no bias.")
        return _single_scorer(tx, sx, out_weight, in_weight, weight, 1.0, _bias_tensor(bias, dev),
                              out_weight.shape[0], fused, pair=target_val is source_val)
    prefix, base = "multihead_", "_low_rank_bilinear"
    agg = kind[len(prefix):-len(base)] if kind.startswith(prefix) and kind.endswith(base) else None
    if agg not in _HEAD_COMBINE:
        raise TypeError(f"Unsupported pairwise kernel kind for b200_sm100a: {kind}")
    if not fused:
        raise TypeError("b200_sm100a multi-head scorers run in the fused kernels only (k <= 64).")
    if in_weight is None or out_weight is None or in_weight.dim() != 3 or out_weight.dim() != 3:
        raise RuntimeError("multi-head projection weights must be [heads, rank, dim].")
    H = in_weight.shape[0]
    row, kph = _multihead_project(tx, out_weight)
    col, _ = _multihead_project(sx, in_weight, core=weight)
    return Scorer(row, col, None, True, heads=Heads(H, kph, _HEAD_COMBINE[agg], _head_bias(bias, H, dev)))


def _route_projections(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                       hidden_weight, hidden_bias, out_weight, out_bias, temperature, src_val, dst_val,
                       fused: bool = True) -> Scorer:
    """Route projections (kernel_common.py:238-295): low_rank_bilinear_route,
    diagonal_bilinear_route or multihead_max_low_rank_bilinear_route; logits =
    (ps . pd + b) / T. Returns a Scorer whose row side is the source (src_proj / T) and
    column side the destination. Other route kinds raise TypeError."""
    if route_kind not in ("low_rank_bilinear_route", "multihead_max_low_rank_bilinear_route",
                          "diagonal_bilinear_route", "full_bilinear_route"):
        raise TypeError(f"Unsupported pairwise route kind for b200_sm100a: {route_kind}")
    temperature = float(temperature)
    if temperature <= 0.0:
        raise RuntimeError("route temperature must be positive.")
    sx, dx = _scorer_input(src_val), _scorer_input(dst_val)
    dev = src_val.device
    if route_kind == "diagonal_bilinear_route":
        if any(t is not None for t in (source_weight, source_bias, target_weight, target_bias, hidden_weight,
                                       hidden_bias, out_weight, out_bias)):
            raise TypeError("Diagonal routes take no projection / hidden layers.")
        sc = _single_scorer(dx, sx, None, None, core_weight, temperature, None, dx.shape[-1], fused)
        return Scorer(sc.col, sc.row, _bias_tensor(bias, dev, temperature), sc.fused, split3=sc.split3)
    if source_weight is None or target_weight is None:
        raise RuntimeError("Low-rank route kernel is missing projection weights.")
    if any(t is not None for t in (source_bias, target_bias, hidden_weight, hidden_bias, out_weight, out_bias)):
        raise TypeError("Low-rank route projections take no bias / hidden layers.")
    if route_kind == "full_bilinear_route":
        # BilinearPairwiseRoute (modules.py:533-564): logits = (src W_s^T) W (dst W_t^T)^T + b, i.e.
        # the source projection against the destination features (dst W_t^T) W^T; f32 features
        # on the select-aggregate path
        ps = _generic_project(sx.reshape(-1, sx.shape[-1]).float(), source_weight, None, temperature)
        with _exact_f32_matmul():
            pd = torch.matmul(_generic_project(dx.reshape(-1, dx.shape[-1]).float(), target_weight),
                              core_weight.detach().float().t())
        return Scorer(ps.reshape(*sx.shape[:-1], -1), pd.reshape(*dx.shape[:-1], -1).contiguous(),
                      _bias_tensor(bias, dev, temperature), False)
    if route_kind == "multihead_max_low_rank_bilinear_route":
        if not fused:
            raise TypeError("b200_sm100a multi-head routes run in the fused kernels only (k <= 64).")
        # max_h(l_h) / T == max_h(l_h / T): every head's source projection and bias take the 1 / T
        H = source_weight.shape[0]
        src_proj, kph = _multihead_project(sx, source_weight, core=core_weight, temperature=temperature)
        dst_proj, _ = _multihead_project(dx, target_weight)
        return Scorer(src_proj, dst_proj, None, True,
                      heads=Heads(H, kph, _lib.JK_HEADS_MAX, _head_bias(bias, H, dev, temperature)))
    sc = _single_scorer(dx, sx, target_weight, source_weight, core_weight, temperature, None,
                        source_weight.shape[0], fused)
    return Scorer(sc.col, sc.row, _bias_tensor(bias, dev, temperature), sc.fused, split3=sc.split3)


# ----------------------------------------------------------------------------- raw kernels
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
    with _on(dev):
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


def select_aggregate(row_f: Tensor, col_f: Tensor, state: Tensor, val: Tensor, k: int, *, window: int = -1,
                     compress: int = _lib.JK_SOFTSIGN, sender: Optional[Tensor] = None,
                     bias: Optional[Tensor] = None, scatter: bool = False, out_dtype: Optional[torch.dtype] = None,
                     return_selection: bool = False, budget: int = _SCORE_BUDGET, score_bias: float = 0.0):
    """Select-aggregate over materialised score blocks (jk_select_aggregate_forward): any k,
    any rank. row_f [B, T, R] and col_f [B, S, R] are the projections (f32, or bf16 / f16
    whose products are exact in f32); every block of rows gets its f32 scores from one GEMM
    (f32 accumulation, TF32 off) and then the exact select / compress / aggregate kernel.

    gather (scatter False): state / sender [B, S], val [B, S, D] per column; returns
    (state [B, T], val [B, T, D]) in out_dtype. scatter True (per-source transition): rows
    are sources with state / sender [B, T], val [B, T, D]; returns the f32 destination sums
    (state [B, S], val [B, S, D]). With return_selection the selected scores (bias
    included) and columns [B, T, min(k, S)] follow, in ascending column order per row."""
    for name, t in (("row_f", row_f), ("col_f", col_f), ("state", state), ("val", val)):
        _require_cuda(name, t)
    B, T, _ = row_f.shape
    S = col_f.shape[1]
    D = val.shape[-1]
    dev = val.device
    kk = max(1, min(int(k), S))
    state = state.contiguous()
    val = val.contiguous()
    snd = None if sender is None else sender.to(state.dtype).contiguous()
    out_dtype = out_dtype or val.dtype
    if scatter:
        acc_state = torch.zeros((B, S), device=dev, dtype=torch.float32)
        acc_val = torch.zeros((B, S, D), device=dev, dtype=torch.float32)
        out_state = out_val = None
    else:
        out_state = torch.empty((B, T), device=dev, dtype=out_dtype)
        out_val = torch.empty((B, T, D), device=dev, dtype=out_dtype)
        acc_state = acc_val = None
    chunk = max(1, min(T, budget // max(1, B * (S + 3 * kk))))
    if return_selection:
        all_s = torch.empty((B, T, kk), device=dev, dtype=torch.float32)
        all_i = torch.empty((B, T, kk), device=dev, dtype=torch.int64)
    sel_s = torch.empty((B, chunk, kk), device=dev, dtype=torch.float32)
    sel_i = torch.empty((B, chunk, kk), device=dev, dtype=torch.int64)
    col_t = col_f.transpose(1, 2)
    with _on(dev):
        for r0 in range(0, T, chunk):
            rc = min(chunk, T - r0)
            if row_f.dtype in (torch.bfloat16, torch.float16):
                # exact products of 16-bit projections, f32 accumulation and output
                sc = torch.bmm(row_f[:, r0:r0 + rc], col_t, out_dtype=torch.float32).contiguous()
            else:
                with _exact_f32_matmul():
                    sc = torch.bmm(row_f[:, r0:r0 + rc], col_t).contiguous()
            check(_LIBRARY.jk_select_aggregate_forward(
                sc.data_ptr(), B, T, S, r0, rc, state.data_ptr(), _ptr(snd), _dtype_code("state", state),
                val.data_ptr(), D, _dtype_code("val", val), kk, int(window), float(score_bias), _ptr(bias), compress,
                1 if scatter else 0, _ptr(out_state), _ptr(out_val), _dtype_code("out", out_state if out_state is not None else val),
                _ptr(acc_state), _ptr(acc_val), sel_s.data_ptr(), sel_i.data_ptr(), _stream(dev)),
                "jk_select_aggregate_forward")
            if return_selection:
                all_s[:, r0:r0 + rc] = sel_s.view(-1)[:B * rc * kk].view(B, rc, kk)
                all_i[:, r0:r0 + rc] = sel_i.view(-1)[:B * rc * kk].view(B, rc, kk)
    res = (acc_state, acc_val) if scatter else (out_state, out_val)
    if return_selection:
        return (*res, all_s, all_i)
    return res


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
    with _on(dev):
        if heads is None:
            check(_LIBRARY.jk_propagation_window_forward(*args, _stream(dev)), "jk_propagation_window_forward")
        else:
            check(_LIBRARY.jk_propagation_window_forward_mh(*args, heads.ref(), _stream(dev)),
                  "jk_propagation_window_forward_mh")
    return out_state, out_val


def _value_planes(pval: Tensor, proj_dtype: torch.dtype):
    """Values for the window-kernel value GEMM: padded to 64 columns. f32 values become bf16
    hi + lo planes (both multiplied by the hi + lo edge planes, ~16 significant bits) unless
    the projections are f16, where they are rounded to f16; 16-bit values are cast to the
    projections' 16-bit type. proj_dtype: torch.float32 for three-plane f32 projections.
    Returns (val, val_lo, pad)."""
    out_dim = pval.shape[-1]
    pad = (-out_dim) % 64
    if pad:
        pval = torch.nn.functional.pad(pval, (0, pad))
    pval_lo = None
    if pval.dtype == torch.float32 and proj_dtype != torch.float16:
        pval = pval.contiguous()
        hi = torch.empty(pval.shape, device=pval.device, dtype=torch.bfloat16)
        pval_lo = torch.empty_like(hi)
        with _on(pval.device):
            check(_LIBRARY.jk_split2_bf16(pval.data_ptr(), pval.numel(), hi.data_ptr(), pval_lo.data_ptr(),
                                          _stream(pval.device)), "jk_split2_bf16")
        pval = hi
    else:
        target = torch.bfloat16 if proj_dtype == torch.float32 else proj_dtype
        if pval.dtype != target:
            pval = pval.to(target)
    return pval.contiguous(), pval_lo, pad


def _split2_bf16(x: Tensor) -> tuple[Tensor, Tensor]:
    """x (f32) = hi + lo as two bf16 planes, one pass (jk_split2_bf16)."""
    x = x.contiguous()
    hi = torch.empty(x.shape, device=x.device, dtype=torch.bfloat16)
    lo = torch.empty_like(hi)
    with _on(x.device):
        check(_LIBRARY.jk_split2_bf16(x.data_ptr(), x.numel(), hi.data_ptr(), lo.data_ptr(), _stream(x.device)),
              "jk_split2_bf16")
    return hi, lo


def _split_stack(x: Tensor, extra: Optional[Tensor], out_cols: int, planes: tuple[int, ...]) -> Tensor:
    """bf16 [B, len(planes) * rows, out_cols]: the planes (0 hi, 1 lo) of f32 x [B, rows, cols]
    (with `extra` [B, rows] as column cols) stacked along the rows (jk_split_stack_bf16)."""
    x = x.contiguous()
    B, rows, cols = x.shape
    out = torch.empty((B, len(planes) * rows, out_cols), device=x.device, dtype=torch.bfloat16)
    bits = sum(p << i for i, p in enumerate(planes))
    with _on(x.device):
        check(_LIBRARY.jk_split_stack_bf16(x.data_ptr(), _ptr(extra), B, rows, cols, out_cols, len(planes), bits,
                                           out.data_ptr(), _stream(x.device)), "jk_split_stack_bf16")
    return out


def routes_aggregate(routes: Tensor, state: Tensor, val: Tensor) -> tuple[Tensor, Tensor]:
    """Aggregate of a dense route matrix: out_state[b, d] = sum_s routes[b, s, d] state[b, s],
    out_val[b, d] = sum_s routes[b, s, d] val[b, s] (f32 results), on the tensor cores with f32
    accumulation and output.
    f32 values: one GEMM. The routes are stacked as bf16 (hi, hi, lo) planes along the source
    dimension and the values, with the state as one more column, as (hi, lo, hi): the GEMM over
    the stacked dimension sums hi.hi + hi.lo + lo.hi (the lo.lo product dropped: ~2^-16
    relative). 16-bit values: the routes split into hi + lo planes of the values' dtype, two
    GEMMs, and the state aggregate as an f32 GEMM."""
    if val.dtype == torch.float32:
        B, S, Dn = routes.shape
        D = val.shape[-1]
        dp = -(-(D + 1) // 8) * 8  # values, state column, zero padding to 16-byte rows
        r3 = _split_stack(routes, None, Dn, (0, 0, 1))
        v3 = _split_stack(val, state.float().contiguous(), dp, (0, 1, 0))
        out = torch.bmm(r3.transpose(1, 2), v3, out_dtype=torch.float32)
        return out[..., D].contiguous(), out[..., :D].contiguous()
    rt = routes.transpose(1, 2)
    with _exact_f32_matmul():
        out_state = torch.bmm(rt, state.float().unsqueeze(-1)).squeeze(-1)
    if val.dtype == torch.float16:
        r_hi = routes.to(torch.float16)
        r_lo = (routes - r_hi.float()).to(torch.float16)
        out_val = torch.bmm(r_hi.transpose(1, 2), val, out_dtype=torch.float32)
        out_val = torch.baddbmm(out_val, r_lo.transpose(1, 2), val, out_dtype=torch.float32)
        return out_state, out_val
    r_hi, r_lo = _split2_bf16(routes)
    out_val = torch.bmm(r_hi.transpose(1, 2), val, out_dtype=torch.float32)
    out_val = torch.baddbmm(out_val, r_lo.transpose(1, 2), val, out_dtype=torch.float32)
    return out_state, out_val


# ----------------------------------------------------------------------------- ops
def _check_edge(edge_compress_name: str) -> int:
    if edge_compress_name not in _EDGE_CODE:
        raise RuntimeError(
            "Only edge_compress_name in {softsign, signed_abs_softmax, signed_entmax15} is supported by the native backend."
        )
    return _EDGE_CODE[edge_compress_name]


def _out_dtype(projected_state: Tensor, projected_val: Tensor) -> torch.dtype:
    return projected_val.dtype if projected_state.dtype == projected_val.dtype else torch.float32


def _propagation_topk_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name,
                           layer_val, projected_state, projected_val, topk: int, window: int):
    compress = _check_edge(edge_compress_name)
    if topk <= 0:
        raise RuntimeError("topk must be positive.")
    for name, t in (("layer_val", layer_val), ("projected_state", projected_state), ("projected_val", projected_val)):
        _require_cuda(name, t)
    n = layer_val.shape[-2]
    k = min(int(topk), n)
    if window < 0 and k >= n:
        # every source survives: the dense propagation (same edges, same sums)
        return _masked_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name,
                            layer_val, layer_val, projected_state, projected_val, -1)
    batch_shape = layer_val.shape[:-2]
    out_dim = projected_val.shape[-1]
    val = _flatten_val(layer_val)
    pstate = _aggregate_input(_flatten_state(projected_state))
    pval = _aggregate_input(_flatten_val(projected_val))
    out_dtype = _out_dtype(projected_state, projected_val)
    sc = _pair_scorer(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, val, val, fused=k <= _MAX_K)
    if sc.fused:
        state, out = topk_aggregate(sc.row, sc.col, pstate, pval, k, window=window, compress=compress, bias=sc.bias,
                                    out_dtype=out_dtype, split3=sc.split3, heads=sc.heads)
    else:
        state, out = select_aggregate(sc.row, sc.col, pstate, pval, k, window=window, compress=compress,
                                      bias=sc.bias, out_dtype=out_dtype)
    return (state.to(projected_state.dtype).reshape(*batch_shape, n),
            out.to(projected_val.dtype).reshape(*batch_shape, n, out_dim))


@_entry
def propagation_topk(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name,
                     layer_val, projected_state, projected_val, topk, target_block_size, source_block_size):
    """SparsePropagation(sparse_type="topk") forward: per target, top-k over every source
    (no causal mask), edges over the k, aggregate. Reference op: jakal_net_native.cpp:6305-6447
    (CUDA fast path :6355-6389, blocked path for any k :6390-6447). Block sizes are accepted
    for signature parity; the kernels tile internally."""
    return _propagation_topk_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias,
                                  edge_compress_name, layer_val, projected_state, projected_val, topk, -1)


@_entry
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


def _transition_inputs(sender_strength, src_val, other_val, projected_state, projected_val):
    for name, t in (("sender_strength", sender_strength), ("src_val", src_val), ("dst/query_val", other_val),
                    ("projected_state", projected_state), ("projected_val", projected_val)):
        _require_cuda(name, t)
    pstate = _aggregate_input(_flatten_state(projected_state))
    sender = _flatten_state(sender_strength).to(pstate.dtype)
    return _flatten_val(src_val), _flatten_val(other_val), pstate, sender, _aggregate_input(_flatten_val(projected_val))


@_entry
def transition_query_topk(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                          hidden_weight, hidden_bias, out_weight, out_bias, temperature, sender_strength, src_val,
                          query_val, projected_state, projected_val, topk, query_block_size, source_block_size,
                          use_cuda_reduce=True):
    """Per-query transition (jakal_net_native.cpp:7089-7246): each query slot takes its
    top-k sources by route logit, softmax over the k, sender-weighted gather."""
    if topk <= 0:
        raise RuntimeError("topk must be positive.")
    sv, qv, pstate, sender, pval = _transition_inputs(sender_strength, src_val, query_val, projected_state,
                                                      projected_val)
    batch_shape = query_val.shape[:-2]
    n_query = query_val.shape[-2]
    n_src = src_val.shape[-2]
    out_dim = projected_val.shape[-1]
    k = min(int(topk), n_src)
    sc = _route_projections(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                            hidden_weight, hidden_bias, out_weight, out_bias, temperature, sv, qv,
                            fused=k <= _MAX_K)
    out_dtype = _out_dtype(projected_state, projected_val)
    # rows = query slots (the route's destination side), columns = sources
    if sc.fused:
        state, out = topk_aggregate(sc.col, sc.row, pstate, pval, k, window=-1, compress=_lib.JK_SOFTMAX,
                                    col_sender=sender, bias=sc.bias, out_dtype=out_dtype, split3=sc.split3,
                                    heads=sc.heads)
    else:
        state, out = select_aggregate(sc.col, sc.row, pstate, pval, k, compress=_lib.JK_SOFTMAX, sender=sender,
                                      bias=sc.bias, out_dtype=out_dtype)
    return (state.to(projected_state.dtype).reshape(*batch_shape, n_query),
            out.to(projected_val.dtype).reshape(*batch_shape, n_query, out_dim))


@_entry
def transition_pairwise_topk(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                             hidden_weight, hidden_bias, out_weight, out_bias, temperature, sender_strength, src_val,
                             dst_val, projected_state, projected_val, topk, src_block_size, dst_block_size,
                             route_compress_name="softmax"):
    """SparseTransition forward (jakal_net_native.cpp:6916-7087): each source takes its
    top-k destinations by route logit, routes compressed over the k, sender-weighted
    scatter-add into the destinations."""
    if topk <= 0:
        raise RuntimeError("topk must be positive.")
    if route_compress_name not in _ROUTE_CODE:
        raise RuntimeError(f"Unsupported route compress {route_compress_name!r}")
    sv, dv, pstate, sender, pval = _transition_inputs(sender_strength, src_val, dst_val, projected_state,
                                                      projected_val)
    batch_shape = src_val.shape[:-2]
    n_dst = dst_val.shape[-2]
    out_dim = projected_val.shape[-1]
    k = min(int(topk), n_dst)
    sc = _route_projections(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                            hidden_weight, hidden_bias, out_weight, out_bias, temperature, sv, dv,
                            fused=k <= _MAX_K)
    compress = _ROUTE_CODE[route_compress_name]
    B = sv.shape[0]
    dev = sv.device
    out_dtype = _out_dtype(projected_state, projected_val)
    if sc.fused and B * sv.shape[1] * n_dst <= _SCORE_BUDGET:
        # routes form: the fused kernel writes the dense route matrix (k non-zeros per source),
        # the aggregate is a GEMM -- no atomics, a fixed summation order
        routes = torch.zeros((B, sv.shape[1], n_dst), device=dev, dtype=torch.float32)
        args = (sc.row.data_ptr(), sc.col.data_ptr(), B, sv.shape[1], n_dst, sc.row.shape[-1],
                _proj_dtype(sc.row, sc.split3), sender.data_ptr(), _dtype_code("sender", sender), k, 0.0,
                _ptr(sc.bias), compress, routes.data_ptr(), None, None)
        with _on(dev):
            if sc.heads is None:
                check(_LIBRARY.jk_transition_pairwise_topk_routes(*args, _stream(dev)),
                      "jk_transition_pairwise_topk_routes")
            else:
                check(_LIBRARY.jk_transition_pairwise_topk_routes_mh(*args, sc.heads.ref(), _stream(dev)),
                      "jk_transition_pairwise_topk_routes_mh")
        out_state, out_val = routes_aggregate(routes, pstate, pval)
    elif sc.fused:
        accum = torch.empty(B * n_dst * (out_dim + 1) + 4, device=dev, dtype=torch.float32)
        out_state = torch.empty((B, n_dst), device=dev, dtype=out_dtype)
        out_val = torch.empty((B, n_dst, out_dim), device=dev, dtype=out_dtype)
        args = (sc.row.data_ptr(), sc.col.data_ptr(), B, sv.shape[1], n_dst, sc.row.shape[-1],
                _proj_dtype(sc.row, sc.split3),
                pstate.data_ptr(), sender.data_ptr(), _dtype_code("state", pstate),
                pval.data_ptr(), out_dim, _dtype_code("val", pval),
                k, 0.0, _ptr(sc.bias), compress, accum.data_ptr(),
                out_state.data_ptr(), out_val.data_ptr(), _dtype_code("out", out_state))
        with _on(dev):
            if sc.heads is None:
                check(_LIBRARY.jk_transition_pairwise_topk_forward(*args, _stream(dev)),
                      "jk_transition_pairwise_topk_forward")
            else:
                check(_LIBRARY.jk_transition_pairwise_topk_forward_mh(*args, sc.heads.ref(), _stream(dev)),
                      "jk_transition_pairwise_topk_forward_mh")
    else:
        out_state, out_val = select_aggregate(sc.row, sc.col, pstate, pval, k, compress=compress, sender=sender,
                                              bias=sc.bias, scatter=True)
    return (out_state.to(projected_state.dtype).reshape(*batch_shape, n_dst),
            out_val.to(projected_val.dtype).reshape(*batch_shape, n_dst, out_dim))


@_entry
def transition_pairwise_dense(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                              hidden_weight, hidden_bias, out_weight, out_bias, route_compress_name, temperature,
                              sender_strength, src_val, dst_val, projected_state, projected_val, src_block_size,
                              dst_block_size):
    """Dense pairwise Transition forward (jakal_net_native.cpp:6705-6914; transition.py:238-254):
    routes of every source compressed over all destinations, sender-weighted, accumulated into
    the destinations. Fused: two launches (per-source route statistics, then the
    per-destination aggregate with per-column normalisation); otherwise the select-aggregate
    kernel's scatter with every destination selected."""
    if route_compress_name not in _ROUTE_CODE:
        raise RuntimeError(f"Unsupported route compress {route_compress_name!r}")
    sv, dv, pstate, sender, pval0 = _transition_inputs(sender_strength, src_val, dst_val, projected_state,
                                                       projected_val)
    batch_shape = src_val.shape[:-2]
    n_src = src_val.shape[-2]
    n_dst = dst_val.shape[-2]
    out_dim = projected_val.shape[-1]
    sc = _route_projections(route_kind, source_weight, source_bias, target_weight, target_bias, core_weight, bias,
                            hidden_weight, hidden_bias, out_weight, out_bias, temperature, sv, dv)
    compress = _ROUTE_CODE[route_compress_name]
    if sc.heads is not None and sc.heads.struct.heads > 2:
        raise TypeError("b200_sm100a dense multi-head routes support 2 heads.")
    out_dtype = _out_dtype(projected_state, projected_val)
    if not sc.fused:
        out_state, out_val = select_aggregate(sc.row, sc.col, pstate, pval0, n_dst, compress=compress,
                                              sender=sender, bias=sc.bias, scatter=True)
        return (out_state.to(projected_state.dtype).reshape(*batch_shape, n_dst),
                out_val.to(projected_val.dtype).reshape(*batch_shape, n_dst, out_dim))
    pval, pval_lo, pad = _value_planes(pval0, torch.float32 if sc.split3 else sc.row.dtype)
    B = sv.shape[0]
    dev = sv.device
    stats = torch.empty(B * n_src * 3, device=dev, dtype=torch.float32)
    out_state = torch.empty((B, n_dst), device=dev, dtype=out_dtype)
    out_val = torch.empty((B, n_dst, pval.shape[-1]), device=dev, dtype=out_dtype)
    args = (sc.row.data_ptr(), sc.col.data_ptr(), B, n_src, n_dst, sc.row.shape[-1],
            _proj_dtype(sc.row, sc.split3),
            pstate.data_ptr(), sender.data_ptr(), _dtype_code("state", pstate),
            pval.data_ptr(), _ptr(pval_lo), pval.shape[-1],
            0.0, _ptr(sc.bias), compress, stats.data_ptr(),
            out_state.data_ptr(), out_val.data_ptr(), _dtype_code("out", out_state))
    with _on(dev):
        if sc.heads is None:
            check(_LIBRARY.jk_transition_pairwise_dense_forward(*args, _stream(dev)),
                  "jk_transition_pairwise_dense_forward")
        else:
            check(_LIBRARY.jk_transition_pairwise_dense_forward_mh(*args, sc.heads.ref(), _stream(dev)),
                  "jk_transition_pairwise_dense_forward_mh")
    if pad:
        out_val = out_val[..., :out_dim]
    return (out_state.to(projected_state.dtype).reshape(*batch_shape, n_dst),
            out_val.to(projected_val.dtype).reshape(*batch_shape, n_dst, out_dim))


def _masked_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, target_val,
                 source_val, projected_state, projected_val, window: int, source_state=None):
    compress = _check_edge(edge_compress_name)
    for name, t in (("target_val", target_val), ("source_val", source_val), ("projected_state", projected_state),
                    ("projected_val", projected_val)):
        _require_cuda(name, t)
    batch_shape = target_val.shape[:-2]
    n_t = target_val.shape[-2]
    n_s = source_val.shape[-2]
    out_dim = projected_val.shape[-1]
    tv = _flatten_val(target_val)
    sv = tv if source_val is target_val else _flatten_val(source_val)
    pstate = _flatten_state(projected_state)
    pval = _flatten_val(projected_val)
    if source_state is not None and source_state.numel() != 0:
        # edges weighted by the source state (jakal_net_native.cpp:6010-6013) == folding the
        # weight into the aggregated inputs
        ss = _flatten_state(source_state).float()
        pstate = (pstate.float() * ss).to(pstate.dtype)
        pval = (pval.float() * ss[..., None]).to(pval.dtype)
    pstate, pval = _aggregate_input(pstate), _aggregate_input(pval)
    sc = _pair_scorer(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, tv, sv)
    if sc.heads is not None and sc.heads.struct.heads > 2:
        raise TypeError("b200_sm100a window / dense multi-head scorers support 2 heads.")
    out_dtype = _out_dtype(projected_state, projected_val)
    if sc.fused:
        pv, pval_lo, pad = _value_planes(pval, torch.float32 if sc.split3 else sc.row.dtype)
        st, out = masked_aggregate(sc.row, sc.col, pstate, pv, window=window, compress=compress, bias=sc.bias,
                                   out_dtype=out_dtype, split3=sc.split3, col_val_lo=pval_lo, heads=sc.heads)
        if pad:
            out = out[..., :out_dim]
    else:
        st, out = select_aggregate(sc.row, sc.col, pstate, pval, n_s, window=window, compress=compress,
                                   bias=sc.bias, out_dtype=out_dtype)
    return (st.to(projected_state.dtype).reshape(*batch_shape, n_t),
            out.to(projected_val.dtype).reshape(*batch_shape, n_t, out_dim))


@_entry
def propagation_window(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, layer_val,
                       projected_state, projected_val, window, target_block_size, source_block_size):
    """SparsePropagation(sparse_type="window") forward: causal window [t - window, t], edges
    compressed over the visible sources, aggregate (jakal_net_native.cpp:6190-6303;
    propagation.py:453-480)."""
    if window < 0:
        raise RuntimeError("window must be non-negative.")
    return _masked_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, layer_val,
                        layer_val, projected_state, projected_val, int(window))


@_entry
def propagation_dense(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, layer_val,
                      projected_state, projected_val, source_state, target_block_size, source_block_size):
    """Dense Propagation forward: every (target, source) pair (jakal_net_native.cpp:5962-6076;
    propagation.py:207-220)."""
    return _masked_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, layer_val,
                        layer_val, projected_state, projected_val, -1, source_state)


@_entry
def propagation_query_dense(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name,
                            query_val, source_val, projected_state, projected_val, query_block_size,
                            source_block_size):
    """Dense query propagation: query rows score every source row (jakal_net_native.cpp:6078-6188)."""
    return _masked_impl(kind, weight, bias, in_weight, in_bias, out_weight, out_bias, edge_compress_name, query_val,
                        source_val, projected_state, projected_val, -1)


# ----------------------------------------------------------------------------- training ops
# The CUDA entry points the reference's autograd Functions call from the native module
# (native_backend.py:659-667 gates on their names; _LowRankTransitionPairwiseTopK,
# native_backend.py:4408-4601, uses them for the per-source sparse transition, forward and
# backward). Positional signatures and return tuples follow jakal_net_native.cpp:152-190,
# 398-416, 450-478.
_PAIRWISE_TOPK_COMPRESS = {0: _lib.JK_SOFTMAX, 1: _lib.JK_SIGNED_ABS_SOFTMAX, 2: _lib.JK_SIGNED_ENTMAX15}


def _cuda_contig(name: str, t: Tensor) -> Tensor:
    _require_cuda(name, t)
    return t.contiguous()


@_entry
def low_rank_pairwise_topk_forward_cuda(weighted_projected_source, projected_target, weighted_projected_state,
                                        weighted_projected_val, topk, score_bias, compress_kind):
    """Per-source top-k transition over given projections (jakal_net_native_cuda.cu:2420-2542
    contract): logits[b, s, d] = wps[b, s] . pt[b, d] + score_bias; every source keeps its
    top-k destinations, routes = compress_kind (0 softmax, 1 signed_abs_softmax,
    2 signed_entmax15) over the k, and scatters routes * wstate / routes * wval.
    Returns (delta_state f32 [B, D], delta_val f32 [B, D, V], topk_scores f32 [B, S, k]
    (score + bias), topk_indices int64 [B, S, k]). 16-bit projections (k <= 64, rank <= 128):
    the fused kernel in routes form, selection in score order, aggregate as GEMMs; otherwise
    the select-aggregate path, selection in destination order (the backward only needs the
    (score, index) pairs)."""
    if weighted_projected_source.dim() != 3:
        raise TypeError("b200_sm100a low_rank_pairwise_topk_forward_cuda takes single-head [B, S, R] projections.")
    if int(compress_kind) not in _PAIRWISE_TOPK_COMPRESS:
        raise RuntimeError(f"unsupported compress kind {compress_kind}")
    wps = _cuda_contig("weighted_projected_source", weighted_projected_source)
    pt = _cuda_contig("projected_target", projected_target).to(wps.dtype)
    if wps.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise RuntimeError(f"unsupported projection dtype {wps.dtype}")
    wstate = _cuda_contig("weighted_projected_state", weighted_projected_state).float()
    wval = _cuda_contig("weighted_projected_val", weighted_projected_val).float()
    k = min(int(topk), pt.shape[1])
    if k <= 0:
        raise RuntimeError("topk must be positive.")
    compress = _PAIRWISE_TOPK_COMPRESS[int(compress_kind)]
    B, S, R = wps.shape
    Dn = pt.shape[1]
    if wps.dtype in (torch.bfloat16, torch.float16) and k <= _MAX_K and R <= 128 and B * S * Dn <= _SCORE_BUDGET:
        # fused kernel in routes form (selection written out), aggregate as GEMMs
        rp = int(_LIBRARY.jk_padded_rank(R))
        if rp != R:
            wps = torch.nn.functional.pad(wps, (0, rp - R))
            pt = torch.nn.functional.pad(pt, (0, rp - R))
        routes = torch.zeros((B, S, Dn), device=wps.device, dtype=torch.float32)
        scores = torch.empty((B, S, k), device=wps.device, dtype=torch.float32)
        index = torch.empty((B, S, k), device=wps.device, dtype=torch.int64)
        with _on(wps.device):
            check(_LIBRARY.jk_transition_pairwise_topk_routes(
                wps.data_ptr(), pt.data_ptr(), B, S, Dn, rp, _DTYPE_CODE[wps.dtype], None, _lib.JK_F32, k,
                float(score_bias), None, compress, routes.data_ptr(), scores.data_ptr(), index.data_ptr(),
                _stream(wps.device)), "jk_transition_pairwise_topk_routes")
        d_state, d_val = routes_aggregate(routes, wstate, wval)
        return d_state, d_val, scores, index
    d_state, d_val, scores, index = select_aggregate(wps, pt, wstate, wval, k, compress=compress, scatter=True,
                                                     return_selection=True, score_bias=float(score_bias))
    return d_state, d_val, scores, index


@_entry
def softmax_backward_cuda(routes, grad_routes):
    """grad_scores = routes * (grad_routes - sum(routes * grad_routes, -1)) (jk_softmax_backward)."""
    r = _cuda_contig("routes", routes)
    g = _cuda_contig("grad_routes", grad_routes).to(r.dtype)
    out = torch.empty_like(r)
    n = r.shape[-1] if r.dim() else 1
    with _on(r.device):
        check(_LIBRARY.jk_softmax_backward(r.data_ptr(), g.data_ptr(), out.data_ptr(), r.numel() // max(n, 1), n,
                                           _dtype_code("routes", r), _stream(r.device)), "jk_softmax_backward")
    return out


@_entry
def softsign_backward_cuda(scores, grad_edges):
    """grad_scores = grad_edges / (1 + |scores|)^2 (jk_softsign_backward)."""
    s = _cuda_contig("scores", scores)
    g = _cuda_contig("grad_edges", grad_edges).to(s.dtype)
    out = torch.empty_like(s)
    with _on(s.device):
        check(_LIBRARY.jk_softsign_backward(s.data_ptr(), g.data_ptr(), out.data_ptr(), s.numel(),
                                            _dtype_code("scores", s), _stream(s.device)), "jk_softsign_backward")
    return out


def _dense_from_topk(w: Tensor, index: Tensor, n_cols: int) -> Tensor:
    """[..., rows, k] weights at int64 columns -> dense f32 [..., rows, n_cols] (jk_topk_to_dense)."""
    w = w.float().contiguous()
    index = index.contiguous()
    dense = torch.zeros(w.shape[:-1] + (n_cols,), device=w.device, dtype=torch.float32)
    with _on(w.device):
        check(_LIBRARY.jk_topk_to_dense(w.data_ptr(), index.data_ptr(), dense.data_ptr(), w.numel() // w.shape[-1],
                                        w.shape[-1], n_cols, _stream(w.device)), "jk_topk_to_dense")
    return dense


@_entry
def query_topk_reduce_backward_cuda(edges, indices, projected_state, projected_val, grad_delta_state, grad_delta_val):
    """Backward of the top-k reduce out[b, q] = sum_e edges[b, q, e] x[b, indices[b, q, e]]
    (jakal_net_native.cpp:152-166 contract). Returns (grad_edges [B, Q, k],
    grad_projected_state [B, S], grad_projected_val [B, S, D]) in the dtype of
    projected_state. The edge gradients are gathered by jk_topk_reduce_backward_edges; the
    source gradients are GEMMs of the dense edge matrix (fixed summation order)."""
    e = _cuda_contig("edges", edges)
    idx = _cuda_contig("indices", indices).long()
    dt = projected_state.dtype
    st = _cuda_contig("projected_state", projected_state)
    B, S = st.reshape(-1, st.shape[-1]).shape
    Q, k = e.shape[-2], e.shape[-1]
    st = st.reshape(B, S)
    vv = _cuda_contig("projected_val", projected_val).to(dt).reshape(B, S, -1)
    D = vv.shape[-1]
    gs = _cuda_contig("grad_delta_state", grad_delta_state).to(dt).reshape(B, Q)
    gv = _cuda_contig("grad_delta_val", grad_delta_val).to(dt).reshape(B, Q, D)
    idx = idx.reshape(B, Q, k)
    grad_edges = torch.empty((B, Q, k), device=e.device, dtype=dt)
    with _on(e.device):
        check(_LIBRARY.jk_topk_reduce_backward_edges(idx.data_ptr(), st.data_ptr(), vv.data_ptr(), gs.data_ptr(),
                                                     gv.data_ptr(), grad_edges.data_ptr(), B, Q, S, k, D,
                                                     _dtype_code("state", st), _dtype_code("out", grad_edges),
                                                     _stream(e.device)), "jk_topk_reduce_backward_edges")
    dense_t = _dense_from_topk(e.reshape(B, Q, k), idx, S).transpose(1, 2)  # [B, S, Q]
    with _exact_f32_matmul():
        g_state = torch.bmm(dense_t, gs.float().unsqueeze(-1)).squeeze(-1)
        g_val = torch.bmm(dense_t, gv.float())
    return (grad_edges.reshape(e.shape), g_state.to(dt).reshape(projected_state.shape),
            g_val.to(dt).reshape(projected_val.shape))


@_entry
def low_rank_pairwise_topk_backward_cuda(src_val, dst_val, target_weight, source_weight, core_weight,
                                         projected_source, projected_target, indices, grad_scores, temperature):
    """Gradient of the low-rank route logits of a per-source top-k transition (the positional
    contract native_backend.py:4559-4570 calls): logits[b, s, e] = (ps[b, s] * core / T) .
    pt[b, indices[b, s, e]] + bias with ps = src_val . W_s^T, pt = dst_val . W_t^T.
    Returns (grad_src_val, grad_dst_val, grad_W_t, grad_W_s, grad_core, grad_bias).
    The sparse grad_scores become a dense [B, S, D] matrix (jk_topk_to_dense), so every
    contraction is a GEMM with f32 accumulation and a fixed summation order."""
    T = float(temperature)
    src = _cuda_contig("src_val", src_val).float()
    dst = _cuda_contig("dst_val", dst_val).float()
    ps = _cuda_contig("projected_source", projected_source).float()
    pt = _cuda_contig("projected_target", projected_target).float()
    c = core_weight.detach().float().reshape(-1)
    w_t = target_weight.detach().float()
    w_s = source_weight.detach().float()
    G = _cuda_contig("grad_scores", grad_scores).float()
    B, S, _ = ps.shape
    Dn = pt.shape[1]
    dense = _dense_from_topk(G, _cuda_contig("indices", indices).long(), Dn)  # [B, S, Dn]
    with _exact_f32_matmul():
        g_wps = torch.bmm(dense, pt)                          # d logits / d (ps * c / T)
        g_pt = torch.bmm(dense.transpose(1, 2), ps * (c / T))  # [B, Dn, R]
        g_ps = g_wps * (c / T)
        g_core = (g_wps * ps).sum(dim=(0, 1)) / T
        grad_src = torch.matmul(g_ps, w_s)
        grad_dst = torch.matmul(g_pt, w_t)
        grad_ws = g_ps.reshape(-1, g_ps.shape[-1]).t() @ src.reshape(-1, src.shape[-1])
        grad_wt = g_pt.reshape(-1, g_pt.shape[-1]).t() @ dst.reshape(-1, dst.shape[-1])
    grad_bias = G.sum()
    return (grad_src.to(src_val.dtype), grad_dst.to(dst_val.dtype), grad_wt.to(target_weight.dtype),
            grad_ws.to(source_weight.dtype), g_core.to(core_weight.dtype).reshape(core_weight.shape),
            grad_bias.to(core_weight.dtype))


def _projected_propagation(weighted_projected_source, projected_target, projected_state, projected_val, *,
                           k: Optional[int], window: int, score_bias: float, compress: int):
    """A propagation over given projections (the contract of the reference's
    low_rank_propagation_*_forward_cuda entry points, jakal_net_native_cuda.cu:2545-3350):
    score[b, t, s] = projected_target[b, t] . wps[b, s] + score_bias, causal window (or none),
    top-k (k None: every visible source), edges, f32 aggregate of f32 state / values.
    16-bit projections of rank <= 128 take the fused kernels; f32 projections the exact
    select-aggregate path."""
    wps = _cuda_contig("weighted_projected_source", weighted_projected_source)
    pt = _cuda_contig("projected_target", projected_target).to(wps.dtype)
    if wps.dim() != 3:
        raise TypeError("b200_sm100a propagation entry points take single-head [B, N, R] projections.")
    st = _cuda_contig("projected_state", projected_state).float()
    vv = _cuda_contig("projected_val", projected_val).float()
    B, N, R = wps.shape
    sb = torch.full((1,), float(score_bias), device=wps.device, dtype=torch.float32)
    n_k = N if k is None else min(int(k), N)
    fused = wps.dtype in (torch.bfloat16, torch.float16) and R <= 128
    if fused:
        rp = int(_LIBRARY.jk_padded_rank(R))
        if rp != R:
            wps = torch.nn.functional.pad(wps, (0, rp - R))
            pt = torch.nn.functional.pad(pt, (0, rp - R))
        if k is not None and n_k <= _MAX_K:
            return topk_aggregate(pt, wps, st, vv, n_k, window=window, compress=compress, bias=sb,
                                  out_dtype=torch.float32)
        if k is None:
            pv, pv_lo, pad = _value_planes(vv, wps.dtype)
            out_s, out_v = masked_aggregate(pt, wps, st, pv, window=window, compress=compress, bias=sb,
                                            out_dtype=torch.float32, col_val_lo=pv_lo)
            return out_s, (out_v[..., :vv.shape[-1]] if pad else out_v)
    return select_aggregate(pt.float() if not fused else pt, wps.float() if not fused else wps, st, vv, n_k,
                            window=window, compress=compress, bias=sb, out_dtype=torch.float32)


_PROP_TOPK_COMPRESS = {0: _lib.JK_SOFTSIGN, 1: _lib.JK_SIGNED_ABS_SOFTMAX, 2: _lib.JK_SIGNED_ENTMAX15}


@_entry
def low_rank_propagation_topk_forward_cuda(weighted_projected_source, projected_target, projected_state,
                                           projected_val, topk, score_bias, compress_kind):
    """Top-k propagation over given projections (native_backend.py:4840-4857 contract,
    jakal_net_native_cuda.cu:2545-2660): per target, the top-k sources over every source (no
    mask), edges compress_kind (0 softsign, 1 signed_abs_softmax, 2 signed_entmax15),
    f32 (delta_state [B, N], delta_val [B, N, D])."""
    if int(compress_kind) not in _PROP_TOPK_COMPRESS:
        raise RuntimeError(f"unsupported compress kind {compress_kind}")
    return _projected_propagation(weighted_projected_source, projected_target, projected_state, projected_val,
                                  k=int(topk), window=-1, score_bias=score_bias,
                                  compress=_PROP_TOPK_COMPRESS[int(compress_kind)])


@_entry
def low_rank_propagation_window_forward_cuda(weighted_projected_source, projected_target, projected_state,
                                             projected_val, window, score_bias):
    """Causal-window softsign propagation over given projections (native_backend.py:5205-5212
    contract, jakal_net_native_cuda.cu:2926): every source in [t - window, t]."""
    return _projected_propagation(weighted_projected_source, projected_target, projected_state, projected_val,
                                  k=None, window=int(window), score_bias=score_bias, compress=_lib.JK_SOFTSIGN)


@_entry
def low_rank_propagation_window_signed_abs_forward_cuda(weighted_projected_source, projected_target,
                                                        projected_state, projected_val, window, score_bias):
    """Causal-window signed_abs_softmax propagation over given projections
    (native_backend.py:5195-5202 contract): edges normalised over each row's visible sources."""
    return _projected_propagation(weighted_projected_source, projected_target, projected_state, projected_val,
                                  k=None, window=int(window), score_bias=score_bias,
                                  compress=_lib.JK_SIGNED_ABS_SOFTMAX)


@_entry
def low_rank_propagation_causal_dense_signed_abs_forward_cuda(weighted_projected_source, projected_target,
                                                              projected_state, projected_val, score_bias):
    """Causal-dense (window N - 1) signed_abs_softmax propagation over given projections
    (native_backend.py:5187-5193 contract)."""
    n = int(projected_target.shape[-2])
    return _projected_propagation(weighted_projected_source, projected_target, projected_state, projected_val,
                                  k=None, window=max(n - 1, 0), score_bias=score_bias,
                                  compress=_lib.JK_SIGNED_ABS_SOFTMAX)


# ----------------------------------------------------------------------------- node routes
def _node_route_features(kind, in_weight, in_bias, out_weight, out_bias, src: Tensor):
    """Route logits over a fixed set of destination nodes (route_kernel_spec,
    kernel_common.py:214-232): linear (logits = src W^T + b) or mlp (logits =
    silu(src W1^T + b1) W2^T + b2), written as the product of per-source features [h, 1]
    and per-destination columns [W, b] so the select-aggregate kernel scores them. Returns
    (row features [B, S, F + 1], destination columns [Dst, F + 1]) in f32."""
    if kind not in ("linear", "mlp"):
        raise TypeError(f"Unsupported route kind for b200_sm100a: {kind}")
    x = src.float()
    with _exact_f32_matmul():
        if kind == "mlp":
            if out_weight is None:
                raise RuntimeError("MLP route kernel is missing its output layer.")
            h = torch.matmul(x, in_weight.detach().float().t())
            if in_bias is not None:
                h = h + in_bias.detach().float()
            h = torch.nn.functional.silu(h)
            w, b = out_weight.detach().float(), out_bias
        else:
            h, w, b = x, in_weight.detach().float(), in_bias
    ones = torch.ones(h.shape[:-1] + (1,), device=h.device, dtype=h.dtype)
    bias = b.detach().float().reshape(-1, 1) if b is not None else torch.zeros((w.shape[0], 1), device=w.device)
    return torch.cat([h, ones], -1).contiguous(), torch.cat([w, bias], -1).contiguous()


def _node_transition(kind, in_weight, in_bias, out_weight, out_bias, compress, sender_strength, src_val,
                     projected_state, projected_val, dst_nodes, k):
    for name, t in (("sender_strength", sender_strength), ("src_val", src_val), ("projected_state", projected_state),
                    ("projected_val", projected_val)):
        _require_cuda(name, t)
    batch_shape = src_val.shape[:-2]
    out_dim = projected_val.shape[-1]
    sv = _flatten_val(src_val)
    pstate = _flatten_state(projected_state)
    pval = _flatten_val(projected_val)
    sender = _flatten_state(sender_strength).to(pstate.dtype)
    rows, cols = _node_route_features(kind, in_weight, in_bias, out_weight, out_bias, sv)
    if cols.shape[0] != int(dst_nodes):
        raise RuntimeError(f"route produces {cols.shape[0]} destinations, expected {dst_nodes}")
    cols = cols.unsqueeze(0).expand(sv.shape[0], -1, -1).contiguous()
    st, vv = select_aggregate(rows, cols, pstate, pval, min(int(k), int(dst_nodes)), compress=compress,
                              sender=sender, scatter=True)
    return (st.to(projected_state.dtype).reshape(*batch_shape, int(dst_nodes)),
            vv.to(projected_val.dtype).reshape(*batch_shape, int(dst_nodes), out_dim))


@_entry
def transition_dense(kind, in_weight, in_bias, out_weight, out_bias, route_compress_name, sender_strength, src_val,
                     projected_state, projected_val, dst_nodes, src_block_size, dst_block_size):
    """Dense Transition with a node route (LinearRoute / MLPRoute; jakal_net_native.cpp
    transition_dense, transition.py:238-254): every source's routes over all destinations,
    compressed, sender-weighted, summed into the destinations (select-aggregate kernel,
    every destination selected)."""
    if route_compress_name not in _ROUTE_CODE:
        raise RuntimeError(f"Unsupported route compress {route_compress_name!r}")
    return _node_transition(kind, in_weight, in_bias, out_weight, out_bias, _ROUTE_CODE[route_compress_name],
                            sender_strength, src_val, projected_state, projected_val, dst_nodes, dst_nodes)


@_entry
def transition_topk(kind, in_weight, in_bias, out_weight, out_bias, sender_strength, src_val, projected_state,
                    projected_val, dst_nodes, topk, src_block_size, dst_block_size):
    """Sparse Transition with a node route (transition_topk_native, native_backend.py:5825-5855):
    each source's top-k destinations, softmax over the k, sender-weighted scatter."""
    if topk <= 0:
        raise RuntimeError("topk must be positive.")
    return _node_transition(kind, in_weight, in_bias, out_weight, out_bias, _lib.JK_SOFTMAX, sender_strength,
                            src_val, projected_state, projected_val, dst_nodes, topk)
