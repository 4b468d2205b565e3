"""ctypes binding of libmoe_b200.so (the C ABI in include/moe_b200.h).

There is no fallback: if the shared library is missing or fails to load, every
entry point raises.  Build it with ``python -m doantotnghiepmoe_b200.build``
or ``__graft_entry__.build()``.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libmoe_b200.so")

MOE_OK = 0
MOE_ERR_INVALID = 1
MOE_ERR_NONFINITE = 2
MOE_ERR_CUDA = 3
MOE_ERR_NCCL = 4
MOE_ERR_TIMEOUT = 5
MOE_ERR_STATE = 6
MOE_ERR_NOMEM = 7
STATUS_NAMES = {0: "OK", 1: "INVALID", 2: "NONFINITE", 3: "CUDA", 4: "NCCL", 5: "TIMEOUT",
                6: "STATE", 7: "NOMEM"}

MOE_ROUTER_F32, MOE_ROUTER_BF16 = 0, 1
MOE_ROUTE_SOFTMAX_TOPK, MOE_ROUTE_TOPK_SOFTMAX = 0, 1
MOE_PATH_AUTO, MOE_PATH_GEMV, MOE_PATH_TENSOR, MOE_PATH_GEMV_PHASED = 0, 1, 2, 3
MOE_PATH_GEMV_FUSED = 4
MOE_PATH_DIGITS = 5
MOE_QUANT_INT8, MOE_QUANT_INT4 = 0, 1

# Every symbol the header declares, with (restype, argtypes).
P, SZ, I32, U32, U64, F32 = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32,
                             ctypes.c_uint64, ctypes.c_float)
PP = ctypes.POINTER(ctypes.c_void_p)


class MoeDims(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("num_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
                ("norm_topk_prob", ctypes.c_int32), ("max_tokens", ctypes.c_int32),
                ("num_layers", ctypes.c_int32)]


class MoeKernelTime(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_int32),
                ("total_ms", ctypes.c_float)]


SIGNATURES = {
    "moe_expert_kernels_init": (I32, [I32, SZ, SZ, SZ, PP]),
    "moe_expert_forward_pairs": (I32, [P, PP, PP, P, P, SZ, PP, SZ, PP]),
    "moe_expert_forward": (I32, [P, PP, PP, P, P, SZ, P, PP]),
    "moe_expert_kernels_max_experts": (SZ, [P]),
    "moe_expert_kernels_last_error": (ctypes.c_char_p, [P]),
    "moe_expert_kernels_destroy": (None, [P]),
    "moe_create": (I32, [I32, ctypes.POINTER(MoeDims), PP]),
    "moe_destroy": (None, [P]),
    "moe_last_error": (ctypes.c_char_p, [P]),
    "moe_set_stream": (I32, [P, P]),
    "moe_set_route_mode": (I32, [P, I32]),
    "moe_set_path": (I32, [P, I32]),
    "moe_set_layer": (I32, [P, I32, PP, PP, P, I32]),
    "moe_set_layer_q": (I32, [P, I32, PP, PP, P, I32, I32]),
    "moe_set_layer_packed": (I32, [P, I32, P, P, P, I32]),
    "moe_set_layer_packed_q": (I32, [P, I32, P, P, P, I32, I32]),
    "moe_route": (I32, [P, I32, P, I32, P, P, P, P]),
    "moe_route_permute": (I32, [P, I32, P, I32, P, P, P, P, P, P]),
    "moe_layer_forward": (I32, [P, I32, P, P, P, I32, P, P, P]),
    "moe_stack_forward": (I32, [P, I32, I32, P, I32, F32, P]),
    "moe_layer_forward_host": (I32, [P, I32, P, P, P, I32, P, P]),
    "moe_ckpt_open": (I32, [ctypes.c_char_p, PP, ctypes.c_char_p, SZ]),
    "moe_ckpt_close": (None, [P]),
    "moe_ckpt_num_tensors": (I32, [P]),
    "moe_ckpt_tensor_info": (I32, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int),
                                   ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64),
                                   ctypes.POINTER(ctypes.c_size_t)]),
    "moe_ckpt_read": (I32, [P, ctypes.c_char_p, P, SZ]),
    "moe_load_layer": (I32, [P, P, I32, I32, I32]),
    "moe_set_layer_norm": (I32, [P, I32, P]),
    "moe_host_alloc": (I32, [SZ, PP]),
    "moe_host_free": (I32, [P]),
    "moe_sync_status": (I32, [P, P]),
    "moe_last_launch_count": (I32, [P]),
    "moe_synth_expert": (I32, [U64, I32, I32, I32, I32, P, P, P]),
    "moe_debug_expf": (I32, [U32, U32, P, P]),
    "moe_profile_enable": (I32, [P, I32]),
    "moe_profile_read": (I32, [P, P, I32, ctypes.POINTER(ctypes.c_int)]),
    "moe_synth_normal_host": (I32, [U64, U32, U32, SZ, F32, P]),
    "moe_layer_forward_noalloc": (I32, [ctypes.POINTER(MoeDims), P, P, P, I32, P, P, P, I32,
                                        P, ctypes.c_char_p, SZ]),
    "moe_ep_unique_id": (I32, [P]),
    "moe_ep_init": (I32, [P, I32, I32, P, P]),
    "moe_ep_set_layer": (I32, [P, I32, P, P, P, I32]),
    "moe_ep_layer_forward": (I32, [P, I32, P, P, P, I32, P]),
    "moe_ep_finalize": (I32, [P]),
    "moe_ep_transport": (I32, [P]),
    "moe_set_graphs": (I32, [P, I32]),
    "moe_set_wait_limit": (I32, [P, U64]),
    "moe_debug_wait_flag": (I32, [P, P]),
    "moe_debug_stream_read": (I32, [P, SZ, P, P]),
}

_lib = None


class MoeError(RuntimeError):
    """A non-OK moe_status, with the library's message (the Rust `Err(String)`)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"CUDA library not built: {LIB_PATH} is missing "
                               "(run python -m doantotnghiepmoe_b200.build)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr_array(values) -> ctypes.Array:
    arr = (ctypes.c_void_p * max(1, len(values)))()
    for i, v in enumerate(values):
        arr[i] = v
    return arr
