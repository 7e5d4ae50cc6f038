"""ctypes binding of libjakal_b200.so (the C ABI declared in include/jakal_b200.h).

The library is built in-tree (``python jakal-net_b200/build.py``) and loaded from this
package directory. There is no fallback: if the library is missing or a call fails, the
error is raised to the caller.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "libjakal_b200.so"
LIB_PATH = Path(os.environ.get("JAKAL_B200_LIB", Path(__file__).resolve().parent / LIB_NAME))

JK_OK = 0
JK_ERR_BAD_SHAPE = -1
JK_ERR_BAD_DTYPE = -2
JK_ERR_UNSUPPORTED_KIND = -3
JK_ERR_UNSUPPORTED_DEVICE = -4
JK_ERR_LAUNCH = -5
JK_ERR_DEVICE_TIMEOUT = -6
JK_ERR_BAD_ARG = -7
JK_ERR_ALIGNMENT = -8

JK_F32, JK_BF16, JK_F16, JK_BF16X3 = 0, 1, 2, 3
JK_SOFTSIGN, JK_SIGNED_ABS_SOFTMAX, JK_SIGNED_ENTMAX15, JK_SOFTMAX = 0, 1, 2, 3

JK_HEADS_MAX, JK_HEADS_SMOOTHMAX, JK_HEADS_SIGNED_SMOOTHMAX = 0, 1, 2


class JkHeads(ctypes.Structure):
    """jk_heads_t: multi-head scorer of the *_mh entry points."""

    _fields_ = [("heads", ctypes.c_int), ("kph", ctypes.c_int), ("combine", ctypes.c_int),
                ("head_bias", ctypes.c_void_p)]


_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes); must list every symbol the header declares.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "jk_status_string": (ctypes.c_char_p, [_i32]),
    "jk_device_check": (_i32, []),
    "jk_device_status": (_i32, [_p, ctypes.POINTER(_i32)]),
    "jk_padded_rank": (_i64, [_i64]),
    "jk_lowrank_project": (_i32, [_p, _i64, _i64, _p, _i64, _p, _f32, _i32, _p, _i64, _p]),
    "jk_lowrank_project_pair": (_i32, [_p, _i64, _i64, _p, _p, _i64, _p, _f32, _i32, _p, _p, _p]),
    "jk_propagation_topk_forward": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i32,  # row_proj, col_proj, B, n_rows, n_cols, rp, proj_dtype
         _p, _p, _i32,                          # col_state, col_sender, state_dtype
         _p, _i64, _i32,                        # col_val, dim, val_dtype
         _i64, _i64, _f32, _p, _i32,            # k, window, score_bias, bias_dev, compress
         _p, _p, _i32, _p, _p, _p],             # out_state, out_val, out_dtype, out_scores, out_index, stream
    ),
    "jk_propagation_window_forward": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i32,  # row_proj, col_proj, B, n_rows, n_cols, rp, proj_dtype
         _p, _i32, _p, _p, _i64,                # col_state, state_dtype, col_val, col_val_lo, dim
         _i64, _f32, _p, _i32,                  # window, score_bias, bias_dev, compress
         _p, _p, _i32, _p],                     # out_state, out_val, out_dtype, stream
    ),
    "jk_transition_pairwise_dense_forward": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i32,  # src_proj, dst_proj, B, n_src, n_dst, rp, proj_dtype
         _p, _p, _i32, _p, _p, _i64,            # src_state, sender, state_dtype, src_val, src_val_lo, dim
         _f32, _p, _i32, _p,                    # score_bias, bias_dev, compress, stats
         _p, _p, _i32, _p],                     # out_state, out_val, out_dtype, stream
    ),
    "jk_split3_bf16": (_i32, [_p, _i64, _i64, _p, _p]),
    "jk_split2_bf16": (_i32, [_p, _i64, _p, _p, _p]),
    "jk_split_stack_bf16": (_i32, [_p, _p, _i64, _i64, _i64, _i64, _i32, ctypes.c_uint, _p, _p]),
    "jk_transition_query_topk_forward": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i32,
         _p, _p, _i32,
         _p, _i64, _i32,
         _i64, _f32, _p, _i32,
         _p, _p, _i32, _p, _p, _p],
    ),
    "jk_transition_pairwise_topk_forward": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i32,
         _p, _p, _i32,
         _p, _i64, _i32,
         _i64, _f32, _p, _i32,
         _p, _p, _p, _i32, _p],
    ),
    "jk_transition_pairwise_topk_forward_noalloc": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i32,
         _p, _p, _i32,
         _p, _i64, _i32,
         _i64, _f32, _p, _i32,
         _p, _p, _i32, _p],
    ),
    "jk_transition_pairwise_topk_noalloc_capacity": (_i64, []),
    "jk_transition_pairwise_topk_routes": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i32,  # src_proj, dst_proj, B, n_src, n_dst, rp, proj_dtype
         _p, _i32, _i64, _f32, _p, _i32,        # src_sender, state_dtype, k, score_bias, bias_dev, compress
         _p, _p, _p, _p],                       # routes, out_scores, out_index, stream
    ),
    "jk_softmax_backward": (_i32, [_p, _p, _p, _i64, _i64, _i32, _p]),
    "jk_softsign_backward": (_i32, [_p, _p, _p, _i64, _i32, _p]),
    "jk_topk_reduce_backward_edges": (
        _i32,
        [_p, _p, _p, _p, _p, _p,                # indices, state, val, grad_state, grad_val, grad_edges
         _i64, _i64, _i64, _i64, _i64,          # B, n_rows, n_src, k, dim
         _i32, _i32, _p],                       # dtype, out_dtype, stream
    ),
    "jk_topk_to_dense": (_i32, [_p, _p, _p, _i64, _i64, _i64, _p]),
    "jk_debug_window_stalled_producer": (
        _i32,
        [_p, _p, _i64, _i64, _i64, _i64, _i32,  # row_proj, col_proj, B, n_rows, n_cols, rp, proj_dtype
         _p, _i32, _p, _i64, _i64,              # col_state, state_dtype, col_val, dim, window
         _p, _p, _i32, _p],                     # out_state, out_val, out_dtype, stream
    ),
    "jk_select_aggregate_forward": (
        _i32,
        [_p, _i64, _i64, _i64, _i64, _i64,      # scores, B, n_rows, n_cols, row_begin, row_count
         _p, _p, _i32, _p, _i64, _i32,          # state, sender, state_dtype, val, dim, val_dtype
         _i64, _i64, _f32, _p, _i32, _i32,      # k, window, score_bias, bias_dev, compress, scatter
         _p, _p, _i32, _p, _p,                  # out_state, out_val, out_dtype, acc_state, acc_val
         _p, _p, _p],                           # sel_score, sel_index, stream
    ),
}
_args = SIGNATURES["jk_propagation_topk_forward"][1]
SIGNATURES["jk_propagation_topk_rows_forward"] = (_i32, _args[:4] + [_i64, _i64] + _args[4:])  # + row block
# The multi-head variants take the same arguments plus a jk_heads_t* before the stream.
_HP = ctypes.POINTER(JkHeads)
for _name in ("jk_propagation_topk_forward", "jk_transition_query_topk_forward", "jk_transition_pairwise_topk_forward",
              "jk_propagation_window_forward", "jk_transition_pairwise_dense_forward",
              "jk_transition_pairwise_topk_routes"):
    _res, _args = SIGNATURES[_name]
    SIGNATURES[_name + "_mh"] = (_res, _args[:-1] + [_HP, _p])

_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads the library once and attaches the declared signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_NAME} not found at {LIB_PATH}; build it with `python jakal-net_b200/build.py`"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


class JakalB200Error(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, where: str):
        self.status = status
        text = load().jk_status_string(status).decode()
        super().__init__(f"{where}: {text} (status {status})")


def check(status: int, where: str) -> None:
    if status != JK_OK:
        raise JakalB200Error(status, where)
