"""ctypes binding of liblitemind_b200.so (the C ABI in include/litemind_moe.h).

The library is built in-tree by ``python -m litemind_b200.build``.  Loading fails
loudly when it is missing: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "liblitemind_b200.so")

LM_OK = 0
LM_ERR_INVALID_ARGUMENT = 1
LM_ERR_CUDA = 2
LM_ERR_NOT_LOADED = 3
LM_ERR_TOO_MANY_TOKENS = 4
LM_ERR_DEVICE_TIMEOUT = 5
LM_ERR_COMM = 6
LM_ERR_UNSUPPORTED = 7

LM_PROFILE_SLOTS = 9
LM_DECODE_TRACE_SLOTS = 16
PROFILE_SLOT_NAMES = ["gather_rows", "route", "router_topk", "dispatch_scan", "place", "gemm_gate_up", "gemm_down",
                      "ep_exchange", "decode_fused"]

LM_DTYPE_UNKNOWN, LM_DTYPE_BF16, LM_DTYPE_F16, LM_DTYPE_F32, LM_DTYPE_OTHER = 0, 1, 2, 3, 4
LM_SAFETENSORS_MAX_DIMS = 8

LM_TOPK_GREEDY = 0
LM_TOPK_GROUP_LIMITED_GREEDY = 1
LM_DEBUG_GRID_EXTRA = 1
LM_DEBUG_WAIT_LIMIT_NS = 2

# Every symbol include/litemind_moe.h declares, with (restype, argtypes).
_vp, _i32, _i64, _f32, _u64p = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.POINTER(C.c_uint64)


class LmMoeConfig(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_int32),
        ("moe_intermediate_size", C.c_int32),
        ("n_routed_experts", C.c_int32),
        ("n_shared_experts", C.c_int32),
        ("num_experts_per_tok", C.c_int32),
        ("norm_topk_prob", C.c_int32),
        ("routed_scaling_factor", C.c_float),
        ("topk_method", C.c_int32),
        ("n_group", C.c_int32),
        ("topk_group", C.c_int32),
        ("rms_norm_eps", C.c_float),
        ("num_layers", C.c_int32),
        ("max_tokens", C.c_int32),
    ]


class LmEpPlan(C.Structure):
    _fields_ = [("send_count", C.c_int32 * 64), ("send_offset", C.c_int32 * 64), ("recv_count", C.c_int32 * 64),
                ("recv_offset", C.c_int32 * 64), ("n_send", C.c_int32), ("n_recv", C.c_int32)]


SIGNATURES = {
    "lm_moe_config_default": (None, [C.POINTER(LmMoeConfig)]),
    "lm_moe_create": (_i32, [C.POINTER(LmMoeConfig), C.c_int, C.POINTER(_vp)]),
    "lm_moe_destroy": (_i32, [_vp]),
    "lm_moe_last_error": (C.c_char_p, [_vp]),
    "lm_status_string": (C.c_char_p, [_i32]),
    "lm_moe_upload_layer": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "lm_moe_upload_expert": (_i32, [_vp, _i32, _i32, _vp, _vp, _vp]),
    "lm_moe_load_safetensors": (_i32, [_vp, _i32, _i32, C.POINTER(C.c_char_p), _i32]),
    "lm_ffn_upload": (_i32, [_vp, _i32, _i32, _vp, _vp, _vp, _vp]),
    "lm_ffn_load_safetensors": (_i32, [_vp, _i32, _i32, _i32, C.POINTER(C.c_char_p), _i32]),
    "lm_ffn_forward": (_i32, [_vp, _i32, _vp, _i32, _vp, _i32, _vp]),
    "lm_ffn_block_forward": (_i32, [_vp, _i32, _vp, _i32, _vp]),
    "lm_safetensors_info": (_i32, [C.c_char_p, C.c_char_p, _vp, _vp, _vp, _vp, _vp, _vp, _i32]),
    "lm_moe_route": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _vp, _vp, _vp]),
    "lm_moe_select": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp]),
    "lm_moe_forward": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _vp]),
    "lm_moe_forward_host": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp]),
    "lm_moe_block_forward": (_i32, [_vp, _i32, _vp, _i32, _vp]),
    "lm_moe_sync": (_i32, [_vp, _vp]),
    "lm_moe_debug_set": (_i32, [_vp, _i32, _i64]),
    "lm_moe_expert_counts": (_i32, [_vp, _vp, _i32]),
    "lm_moe_memory": (_i32, [_vp, _u64p, _u64p]),
    "lm_moe_ep_init": (_i32, [_vp, _vp, _i32, _i32]),
    "lm_moe_ep_unique_id": (_i32, [_vp]),
    "lm_moe_ep_plan": (_i32, [_i32, _i32, _vp, _vp, C.POINTER(LmEpPlan)]),
    "lm_moe_ep_chunk_plan": (_i32, [_i32, _i32, _i32, _i32, _vp, _vp, C.POINTER(LmEpPlan)]),
    "lm_moe_profile_enable": (_i32, [_vp, _i32]),
    "lm_moe_profile_read": (_i32, [_vp, _vp, _vp, _i32]),
    "lm_moe_profile_trace": (_i32, [_vp, _vp, _i32, _vp]),
    "lm_moe_profile_ep_timeline": (_i32, [_vp, _vp, _i32, C.POINTER(C.c_int32)]),
    "lm_moe_route_static": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _vp]),
    "lm_kernel_description": (C.c_char_p, []),
    "lm_gemm_matvec_bf16": (_i32, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "lm_gemm_matvec_bf16_accumulate": (_i32, [_vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "lm_gemm_matvec_f32": (_i32, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "lm_gemm_softmax": (_i32, [_vp, _i64, _i64, _vp]),
    "lm_gemm_silu_multiply": (_i32, [_vp, _vp, _vp, _i64, _vp]),
    "lm_gemm_rms_norm": (_i32, [_vp, _vp, _i64, _i64, _f32, _vp]),
    "lm_gemm_axpy": (_i32, [_f32, _vp, _vp, _i64, _vp]),
}

_lib = None


class LiteMindError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


def load(path: str = LIB_PATH) -> C.CDLL:
    """Opens the library (once) and declares every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is not built; run `python -m litemind_b200.build` (no CPU fallback exists)")
    lib = C.CDLL(path)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def check(status: int, ctx=None) -> None:
    if status != LM_OK:
        lib = load()
        msg = lib.lm_moe_last_error(ctx)
        text = (msg or b"").decode() or lib.lm_status_string(status).decode()
        raise LiteMindError(status, text)
