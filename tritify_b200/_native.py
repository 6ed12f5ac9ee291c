"""ctypes binding of libktmoe.so (the C ABI of include/ktmoe.h).

The library is the product: every integer of a forward comes from its sm_100a kernels. There is no fallback: if the
library is missing or cannot load, importing the binding raises.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libktmoe.so")

OK = 0
ERR_CUDA, ERR_ARG, ERR_RANGE, ERR_KERNEL, ERR_UNSUPPORTED, ERR_NO_DEVICE, ERR_STATE, ERR_CALLBACK = (1, 2, 3, 4, 5,
                                                                                                 6, 7, 8)


class KtmoeScale(ctypes.Structure):
    _fields_ = [("mant", ctypes.c_int64), ("shift", ctypes.c_int32)]


class KtmoeLayerConfig(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_int32),
        ("n_experts", ctypes.c_int32),
        ("d_ff", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("norm_topk_prob", ctypes.c_int32),
        ("router_score", ctypes.c_int32),
        ("shared_d_ff", ctypes.c_int32),
    ]


# Every symbol include/ktmoe.h declares, with its ctypes signature.
_P = ctypes.POINTER
_vp, _i32p, _i64p, _f32p = ctypes.c_void_p, _P(ctypes.c_int32), _P(ctypes.c_int64), _P(ctypes.c_float)
_i64, _u64, _i32 = ctypes.c_int64, ctypes.c_uint64, ctypes.c_int32
SIGNATURES = {
    "ktmoe_device_count": ([_P(ctypes.c_int)], ctypes.c_int),
    "ktmoe_open": ([ctypes.c_int, _P(_vp)], ctypes.c_int),
    "ktmoe_close": ([_vp], ctypes.c_int),
    "ktmoe_error_string": ([ctypes.c_int], ctypes.c_char_p),
    "ktmoe_last_error": ([_vp], ctypes.c_char_p),
    "ktmoe_stream": ([_vp], _vp),
    "ktmoe_linear": ([_vp, _i32p, _i32p, _i64, _i64, _i64, _i64p], ctypes.c_int),
    "ktmoe_linear_weights": ([_vp, _u64, _i32p, _i32p, _i64, _i64, _i64, _i64p], ctypes.c_int),
    "ktmoe_linear_noalloc": ([_i32, _vp, _vp, _i64, _i64, _i64, _vp, _vp], ctypes.c_int),
    "ktmoe_linear_last_gemm": ([_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_i32)], ctypes.c_int),
    "ktmoe_wire_size": ([_i32, _i64, ctypes.POINTER(_u64)], ctypes.c_int),
    "ktmoe_check_wait_expiry": ([_vp], ctypes.c_int),
    "ktmoe_layer_expert_forward": ([_vp, _vp, _i64, KtmoeScale, _vp, _i32, _vp, _vp], ctypes.c_int),
    "ktmoe_layer_forward_with_experts": ([_vp, _vp, _i64, KtmoeScale, _vp, _vp, _vp, _vp], ctypes.c_int),
    "ktmoe_wire_encode": ([_vp, _i64, _vp, _i32, KtmoeScale, _vp, _u64, ctypes.POINTER(_u64)], ctypes.c_int),
    "ktmoe_wire_decode": ([_vp, _u64, ctypes.POINTER(_i32), _vp, _i32, ctypes.POINTER(KtmoeScale), ctypes.POINTER(_i64),
                           _vp, _i64, ctypes.POINTER(_u64)], ctypes.c_int),
    "ktmoe_set_weight_budget": ([_vp, _u64], ctypes.c_int),
    "ktmoe_resident_bytes": ([_vp, _P(_u64)], ctypes.c_int),
    "ktmoe_layer_create": ([_vp, _P(KtmoeLayerConfig), _P(_vp)], ctypes.c_int),
    "ktmoe_ep_unique_id": ([_vp, _i64], ctypes.c_int),
    "ktmoe_layer_create_ep": ([_vp, _P(KtmoeLayerConfig), _i32, _i32, _vp, _P(_vp)], ctypes.c_int),
    "ktmoe_layer_experts": ([_vp, _P(_i32), _P(_i32)], ctypes.c_int),
    "ktmoe_layer_set_ep_capacity": ([_vp, _i64], ctypes.c_int),
    "ktmoe_layer_set_graphs": ([_vp, _i32], ctypes.c_int),
    "ktmoe_layer_set_norm": ([_vp, _i32p, KtmoeScale, KtmoeScale], ctypes.c_int),
    "ktmoe_block_forward": ([_vp, _i32p, _i64, KtmoeScale, _i32p, _P(KtmoeScale)], ctypes.c_int),
    "ktmoe_block_forward_dev": ([_vp, _vp, _i64, _vp, _vp, _vp, _vp], ctypes.c_int),
    "ktmoe_scale_from_f64": ([ctypes.c_double, _P(KtmoeScale)], ctypes.c_int),
    "ktmoe_layer_destroy": ([_vp], ctypes.c_int),
    "ktmoe_layer_set_router": ([_vp, _i32p, KtmoeScale, _i64p, KtmoeScale], ctypes.c_int),
    "ktmoe_layer_set_sigmoid_bias": ([_vp, _i64p], ctypes.c_int),
    "ktmoe_layer_set_expert": ([_vp, _i32, _i32p, KtmoeScale, _i32p, KtmoeScale, _i32p, KtmoeScale], ctypes.c_int),
    "ktmoe_layer_set_shared": ([_vp, _i32p, KtmoeScale, _i32p, KtmoeScale, _i32p, KtmoeScale], ctypes.c_int),
    "ktmoe_layer_set_shared_gate": ([_vp, _i32p, KtmoeScale], ctypes.c_int),
    "ktmoe_forward_async": ([_vp, _i32p, _i64, KtmoeScale, _i32p, ctypes.POINTER(KtmoeScale)], ctypes.c_int),
    "ktmoe_forward_async_wait": ([_vp], ctypes.c_int),
    "ktmoe_layer_set_depth": ([_vp, _i32], ctypes.c_int),
    "ktmoe_layer_select": ([_vp, _i32], ctypes.c_int),
    "ktmoe_layer_synth_weights": ([_vp, _u64, ctypes.c_float, ctypes.c_float, _i32], ctypes.c_int),
    "ktmoe_synth_normal_portable": ([_u64, ctypes.c_float, _u64, _i64, _f32p], ctypes.c_int),
    "ktmoe_synth_normal_portable_dev": ([_vp, _u64, ctypes.c_float, _u64, _i64, _vp], ctypes.c_int),
    "ktmoe_forward": ([_vp, _i32p, _i64, KtmoeScale, _i32p, _P(KtmoeScale)], ctypes.c_int),
    "ktmoe_forward_dev": ([_vp, _vp, _i64, _vp, _vp, _vp, _vp], ctypes.c_int),
    "ktmoe_sync": ([_vp, _vp], ctypes.c_int),
    "ktmoe_route": ([_vp, _i32p, _i64, KtmoeScale, _i32p, _i64p, _i64p], ctypes.c_int),
    "ktmoe_route_margins": ([_i32p, _i64, _i32, _P(KtmoeScale), _i32p, _i32, _P(ctypes.c_double)], ctypes.c_int),
    "ktmoe_launch_count": ([_vp, _P(_u64)], ctypes.c_int),
    "ktmoe_layer_debug_fetch": ([_vp, _i32, _vp, _i64], ctypes.c_int),
    "ktmoe_layer_set_timing": ([_vp, _i32], ctypes.c_int),
    "ktmoe_layer_stage_times": ([_vp, _P(ctypes.c_double), _i32, _P(_i32)], ctypes.c_int),
    "ktmoe_quantize_weights": ([_f32p, _i64, _i32p, _P(KtmoeScale)], ctypes.c_int),
    "ktmoe_quantize_bias": ([_f32p, _i64, _i64p, _P(KtmoeScale), _P(_i32)], ctypes.c_int),
    "ktmoe_code_sigmoid_bias": ([_f32p, _i64, _i64p], ctypes.c_int),
    "ktmoe_from_reals": ([_f32p, _i64, _i32p, _P(KtmoeScale)], ctypes.c_int),
    "ktmoe_table": ([_i32, _i64p, _P(KtmoeScale), _i64p, _P(KtmoeScale)], ctypes.c_int),
    "ktmoe_synth_normal": ([_u64, ctypes.c_float, _u64, _i64, _f32p], ctypes.c_int),
    "ktmoe_lcg_uniform": ([_u64, _i64, _i64, _i64, _i32p], ctypes.c_int),
}

_lib = None


def lib():
    """Load libktmoe.so (raises if it is missing: there is no other implementation to fall back to)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python tritify_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


class KtmoeError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"ktmoe status {status}: {message}")
        self.status = status


# ktmoe_experts_fn: (user, rows, top_k, ids, x, x_scale, y, y_scale) -> int
EXPERTS_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
                              ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32), KtmoeScale,
                              ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(KtmoeScale))


def check(status: int, ctx=None) -> None:
    if status != OK:
        msg = lib().ktmoe_error_string(status).decode()
        if ctx is not None:
            detail = lib().ktmoe_last_error(ctx)
            if detail:
                msg += f" ({detail.decode()})"
        raise KtmoeError(status, msg)
