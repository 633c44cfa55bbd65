"""ctypes binding of ``libmoe_b200.so`` (declared in ``include/moe_b200.h``).

The library is built in tree by ``build.py`` and loaded from this directory;
there is no other implementation to fall back to.  If it is missing, every
entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_b200.so")

MOE_OK = 0
MOE_ERR_INVALID_ARG = -1
MOE_ERR_SHAPE = -2
MOE_ERR_ALIGNMENT = -3
MOE_ERR_WORKSPACE = -4
MOE_ERR_CUDA = -5
MOE_ERR_TIMEOUT = -6
MOE_ERR_DEVICE = -7
MOE_ERR_TOO_LARGE = -8
MOE_ERR_BOUNDS = -9

MOE_PROFILE_EVENTS = 6

# What failed, in bits 24-31 of the info word of MOE_ERR_BOUNDS.
CHECK_SITES = {1: "counts", 2: "tile_start", 3: "topk_idx", 4: "topk_weights", 5: "row_token",
               6: "row_weight", 7: "row_expert", 8: "assign_row", 9: "guard"}

MOE_BIAS_F32 = 0
MOE_BIAS_BF16 = 1
MOE_BIAS_F16 = 2

MOE_FLAG_DETERMINISTIC = 0x1
MOE_FLAG_DEBUG = 0x2
MOE_FLAG_TEST_STALL = 0x100


class MoeFwdArgs(ctypes.Structure):
    _fields_ = [
        ("routing_logits", ctypes.c_void_p),
        ("routing_bias", ctypes.c_void_p),
        ("hidden_states", ctypes.c_void_p),
        ("hidden_states_scale", ctypes.c_void_p),
        ("gemm1_weights", ctypes.c_void_p),
        ("gemm1_weights_scale", ctypes.c_void_p),
        ("gemm2_weights", ctypes.c_void_p),
        ("gemm2_weights_scale", ctypes.c_void_p),
        ("output", ctypes.c_void_p),
        ("T", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("I", ctypes.c_int64),
        ("E_global", ctypes.c_int64),
        ("E_local", ctypes.c_int64),
        ("local_expert_offset", ctypes.c_int64),
        ("n_group", ctypes.c_int64),
        ("topk_group", ctypes.c_int64),
        ("top_k", ctypes.c_int64),
        ("routed_scaling_factor", ctypes.c_float),
        ("bias_dtype", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("flags", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32),
        ("wait_limit_ns", ctypes.c_uint64),
        ("gemm2_weights_bf16", ctypes.c_void_p),
        ("n_shared_experts", ctypes.c_int64),
    ]


class MoeWorkspaceLayout(ctypes.Structure):
    _fields_ = [
        ("total_bytes", ctypes.c_size_t),
        ("npad", ctypes.c_int64),
        ("route_blocks", ctypes.c_int64),
        ("tokens_per_block", ctypes.c_int64),
        ("ctrl", ctypes.c_size_t),
        ("topk_idx", ctypes.c_size_t),
        ("topk_weights", ctypes.c_size_t),
        ("block_base", ctypes.c_size_t),
        ("counts", ctypes.c_size_t),
        ("tile_start", ctypes.c_size_t),
        ("row_token", ctypes.c_size_t),
        ("row_weight", ctypes.c_size_t),
        ("a_perm", ctypes.c_size_t),
        ("a_scale_perm", ctypes.c_size_t),
        ("inter", ctypes.c_size_t),
        ("inter_scale", ctypes.c_size_t),
        ("out_f32", ctypes.c_size_t),
        ("assign_row", ctypes.c_size_t),
        ("rows_out", ctypes.c_size_t),
        ("inter_bf16", ctypes.c_size_t),
    ]


# Every symbol include/moe_b200.h declares, with its ctypes signature.
class MoeEpConfig(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("T_max", ctypes.c_int64),
                ("H", ctypes.c_int64), ("I", ctypes.c_int64), ("E_global", ctypes.c_int64),
                ("n_group", ctypes.c_int64), ("topk_group", ctypes.c_int64),
                ("top_k", ctypes.c_int64)]


_VP = ctypes.c_void_p
SYMBOLS = {
    "moe_fp8_workspace_size": (ctypes.c_int, [ctypes.POINTER(MoeFwdArgs),
                                              ctypes.POINTER(ctypes.c_size_t)]),
    "moe_fp8_workspace_layout": (ctypes.c_int, [ctypes.POINTER(MoeFwdArgs),
                                                ctypes.POINTER(MoeWorkspaceLayout)]),
    "moe_fp8_forward": (ctypes.c_int, [ctypes.POINTER(MoeFwdArgs), ctypes.c_void_p]),
    "moe_fp8_forward_profiled": (ctypes.c_int, [ctypes.POINTER(MoeFwdArgs), ctypes.c_void_p,
                                                ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]),
    "moe_fp8_route": (ctypes.c_int, [ctypes.POINTER(MoeFwdArgs), ctypes.c_void_p]),
    "moe_fp8_device_error": (ctypes.c_int, [ctypes.POINTER(MoeFwdArgs), ctypes.c_void_p,
                                            ctypes.POINTER(ctypes.c_int32),
                                            ctypes.POINTER(ctypes.c_int32)]),
    "moe_router_workspace_size": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                 ctypes.POINTER(ctypes.c_size_t)]),
    "moe_router_logits_bf16": (ctypes.c_int, [_VP, _VP, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64, _VP, _VP, ctypes.c_size_t, _VP]),
    "moe_fp8_check_workspace": (ctypes.c_int, [ctypes.POINTER(MoeFwdArgs), ctypes.c_void_p]),
    "moe_fp8_route_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                             ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_float, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "moe_bf16_to_fp8_1x128": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "moe_fp8_prepare_gemm2_bf16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                                  ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                                  ctypes.c_void_p]),
    "moe_ep_create": (ctypes.c_int, [ctypes.POINTER(MoeEpConfig), ctypes.POINTER(_VP)]),
    "moe_ep_ipc_handle": (ctypes.c_int, [_VP, _VP]),
    "moe_ep_connect": (ctypes.c_int, [_VP, ctypes.c_char_p]),
    "moe_ep_send_plan": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_int32, ctypes.c_int64,
                                        ctypes.c_float, _VP, _VP]),
    "moe_ep_dispatch": (ctypes.c_int, [_VP, _VP, _VP, _VP, ctypes.c_int64, _VP, _VP]),
    "moe_ep_experts": (ctypes.c_int, [_VP, _VP, ctypes.c_int32, ctypes.c_float, _VP, _VP, _VP,
                                      _VP, _VP, _VP]),
    "moe_ep_finalize": (ctypes.c_int, [_VP, ctypes.c_int64, _VP, _VP]),
    "moe_ep_device_error": (ctypes.c_int, [_VP, _VP, ctypes.POINTER(ctypes.c_int32),
                                           ctypes.POINTER(ctypes.c_int32)]),
    "moe_ep_destroy": (ctypes.c_int, [_VP]),
    "moe_fp8_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "moe_fp8_num_sms": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int32)]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the in-tree library once; raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python mlsys26-flashinfer-moe_b200/build.py` (no CPU fallback exists)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SYMBOLS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def status_string(code: int) -> str:
    return load().moe_fp8_status_string(code).decode()


class MoeError(RuntimeError):
    def __init__(self, code: int, where: str):
        super().__init__(f"{where}: {status_string(code)} (status {code})")
        self.code = code
