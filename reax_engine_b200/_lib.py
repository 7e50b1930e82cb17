"""ctypes binding of the C-ABI library (include/reaxmoe.h). No torch types cross this boundary: raw pointers,
ints and a cudaStream_t passed as void*."""
from __future__ import annotations

import ctypes
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libreaxmoe.so")

OK = 0
ERR_BAD_SHAPE = 1
ERR_MISALIGNED = 2
ERR_TOO_MANY_EXPERTS = 3
ERR_DEVICE_TIMEOUT = 4
ERR_WORKSPACE = 5
ERR_CUDA = 6
ERR_NULL = 7
ERR_BAD_EXPERT_ID = 8
ERR_UNSUPPORTED = 9

ACT_SILU = 0
ACT_GELU_TANH = 1

ERROR_NAMES = {
    ERR_BAD_SHAPE: "BAD_SHAPE", ERR_MISALIGNED: "MISALIGNED", ERR_TOO_MANY_EXPERTS: "TOO_MANY_EXPERTS",
    ERR_DEVICE_TIMEOUT: "DEVICE_TIMEOUT", ERR_WORKSPACE: "WORKSPACE", ERR_CUDA: "CUDA", ERR_NULL: "NULL",
    ERR_BAD_EXPERT_ID: "BAD_EXPERT_ID", ERR_UNSUPPORTED: "UNSUPPORTED",
}


class ReaxMoEError(RuntimeError):
    def __init__(self, code: int, text: str):
        super().__init__(f"reaxmoe error {code} ({ERROR_NAMES.get(code, '?')}): {text}")
        self.code = code


class Problem(ctypes.Structure):
    _fields_ = [("tokens", ctypes.c_int32), ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32),
                ("experts", ctypes.c_int32), ("topk", ctypes.c_int32), ("activation", ctypes.c_int32)]


class ForwardArgs(ctypes.Structure):
    _fields_ = [("p", Problem)] + [(n, ctypes.c_void_p) for n in (
        "a", "a1_gscale", "w1_fp4", "w1_sf", "w1_alphas", "a2_gscale", "w2_fp4", "w2_sf", "w2_alphas",
        "topk_weights", "topk_ids", "output")]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_PP = ctypes.POINTER(Problem)

SIGNATURES = {
    "reaxmoe_version": (_I32, []),
    "reaxmoe_last_error": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
    "reaxmoe_workspace_size": (ctypes.c_size_t, [_PP]),
    "reaxmoe_forward": (ctypes.c_int, [ctypes.POINTER(ForwardArgs), _P, ctypes.c_size_t, _P]),
    "reaxmoe_route": (ctypes.c_int, [_P, _P, _I32, _I32, _I32, _P, _P, _P]),
    "reaxmoe_router_topk": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_float, _I32, _I32, _I32, _I32, _P, _P, _P, _P,
                                           _P]),
    "reaxmoe_set_sm_budget": (None, [_I32]),
    "reaxmoe_rmsnorm": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_float, ctypes.c_int64, _I32, _P, _P]),
    "reaxmoe_qkv_norm_rope": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, ctypes.c_float, ctypes.c_int64, _I32, _I32, _I32,
                                             _P, _P, _P, _P]),
    "reaxmoe_gelu_tanh_mul": (ctypes.c_int, [_P, ctypes.c_int64, _I32, _P, _P]),
    "reaxmoe_rmsnorm_nvfp4": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_float, ctypes.c_int64, _I32, ctypes.c_float,
                                             _P, _P, _P, _P]),
    "reaxmoe_forward_prequant": (ctypes.c_int, [ctypes.POINTER(ForwardArgs), _P, ctypes.c_float, _P, ctypes.c_size_t,
                                                _P]),
    "reaxmoe_plan": (ctypes.c_int, [_PP, _P, _P, ctypes.c_size_t, _P, _P, _P, _P, _P]),
    "reaxmoe_permute_quant": (ctypes.c_int, [_PP, _P, _P, _P, _P, ctypes.c_size_t, _P, _P, _P, _P]),
    "reaxmoe_gemm_w13": (ctypes.c_int, [_PP, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P, _P, _P]),
    "reaxmoe_gemm_w2": (ctypes.c_int, [_PP, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P, _P]),
    "reaxmoe_combine": (ctypes.c_int, [_PP, _P, _P, _P, _P, _P]),
    "reaxmoe_quantize": (ctypes.c_int, [_P, _I32, _I64, _I32, _I32, _P, _P, _P, _P]),
    "reaxmoe_prepack_w13": (ctypes.c_int, [_P, _P, _I32, _I32, _I32, _P, _P, _P]),
    "reaxmoe_read_status": (ctypes.c_int, [_P, ctypes.c_size_t, _I32, _P]),
    "reaxmoe_plan_static": (ctypes.c_int, [_PP, _P, _P, _P, _P, _P, _P]),
    "reaxmoe_ep_record_bytes": (ctypes.c_size_t, [_I32, _I32]),
    "reaxmoe_ep_dispatch_workspace_size": (ctypes.c_size_t, [_PP, _I32]),
    "reaxmoe_ep_dispatch": (ctypes.c_int, [_PP, _I32, _P, _P, _P, _P, _P, ctypes.c_size_t, _P, _P, _P, _P]),
    "reaxmoe_ep_expert_workspace_size": (ctypes.c_size_t, [_PP]),
    "reaxmoe_ep_expert_forward": (ctypes.c_int, [_PP, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P,
                                                 _P]),
    "reaxmoe_ep_combine": (ctypes.c_int, [_I32, _I32, _I32, _P, _P, _P, _P]),
    "reaxmoe_ipc_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _P]),
    "reaxmoe_ipc_open": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "reaxmoe_ipc_close": (ctypes.c_int, [_P]),
    "reaxmoe_ipc_free": (ctypes.c_int, [_P]),
    "reaxmoe_ep_signal_bytes": (ctypes.c_size_t, []),
    "reaxmoe_ep_signal": (ctypes.c_int, [_I32, _I32, _P, ctypes.c_uint32, _P, ctypes.c_uint64, _P]),
    "reaxmoe_ep_dispatch_plan": (ctypes.c_int, [_PP, _I32, _P, _P, _P, ctypes.c_size_t, _P, _P]),
    "reaxmoe_ep_dispatch_pack": (ctypes.c_int, [_PP, _I32, _P, _P, _P, _P, _P, ctypes.c_size_t, _P, _P, _P]),
    "reaxmoe_ep_expert_forward_to": (ctypes.c_int, [_PP, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _I32,
                                                    _P, _P, _P]),
    "reaxmoe_ep_expert_gemms": (ctypes.c_int, [_PP, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _I32, _P]),
    "reaxmoe_ep_presum_to": (ctypes.c_int, [_PP, _P, ctypes.c_size_t, _I32, _P, _P, _I32, _P]),
    "reaxmoe_ep_copy_rows": (ctypes.c_int, [_I32, _P, _P, _P, _P]),
}

_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library. Raises if it has not been built: there is no fallback implementation."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m reax_engine_b200._build`")
                h = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = h
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().reaxmoe_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != OK:
        raise ReaxMoEError(rc, last_error())


def problem(tokens: int, hidden: int, inter: int, experts: int, topk: int, activation: int) -> Problem:
    return Problem(tokens, hidden, inter, experts, topk, activation)
