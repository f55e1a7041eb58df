"""ctypes binding of libmoe_sm100.so (declarations: include/moe_sm100.h).

The shared library is built in-tree next to this file (``moe_sm100.build``).
There is no fallback: if the library is missing every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_uint64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmoe_sm100.so")

MOE_OK = 0
MOE_ERR_INVALID = 1
MOE_ERR_CUDA = 2
MOE_ERR_UNSUPPORTED = 3
MOE_ERR_MISSING_TENSOR = 4
MOE_ERR_WORKSPACE = 5
MOE_ERR_NOT_BOUND = 6
MOE_ERR_DEVICE = 7
MOE_ERR_TIMEOUT = 8
MOE_ERR_RANGE = 9

MOE_STATIC_SCRATCH_BYTES = 32 * 1024 * 1024  # include/moe_sm100.h

MOE_SCORE_SOFTMAX = 0
MOE_SCORE_SIGMOID = 1
MOE_WEIGHTS_F16 = 0
MOE_WEIGHTS_INT8_PC = 1


class MoeConfigC(ctypes.Structure):
    _fields_ = [
        ("hidden", c_int32), ("n_experts", c_int32), ("top_k", c_int32), ("inter", c_int32),
        ("shared_inter", c_int32), ("score_func", c_int32), ("norm_topk_prob", c_int32),
        ("use_bias", c_int32), ("has_shared_gate", c_int32), ("weight_format", c_int32),
        ("routed_scaling_factor", c_float), ("rms_norm_eps", c_float), ("max_tokens", c_int32),
        ("expert_begin", c_int32), ("expert_end", c_int32), ("device", c_int32),
    ]


class MoeAttnConfigC(ctypes.Structure):
    _fields_ = [
        ("hidden", c_int32), ("heads", c_int32), ("kv_heads", c_int32), ("head_dim", c_int32),
        ("rotary_dim", c_int32), ("rope_theta", c_float), ("rms_norm_eps", c_float),
        ("max_tokens", c_int32), ("device", c_int32),
    ]


class MoeTensorDescC(ctypes.Structure):
    _fields_ = [
        ("name", c_char_p), ("dtype", c_char_p), ("shape", c_int64 * 2), ("ndim", c_int32),
        ("offset", c_int64), ("nbytes", c_int64),
    ]


class MoeError(RuntimeError):
    """Status returned by libmoe_sm100 (``RuntimeError`` like the reference's ``_check``)."""

    def __init__(self, code: int, message: str) -> None:
        super().__init__(f"moe_sm100 error {code}: {message}")
        self.code = code


class MoeValueError(MoeError, ValueError):
    pass


class MoeKeyError(MoeError, KeyError):
    pass


# name -> (restype, argtypes); kept in the same order as include/moe_sm100.h
_PROTOTYPES: dict[str, tuple] = {
    "moe_plan_create": (c_int32, [POINTER(MoeConfigC), POINTER(c_void_p)]),
    "moe_plan_destroy": (c_int32, [c_void_p]),
    "moe_bind_layer": (c_int32, [c_void_p, c_void_p, c_uint64, POINTER(MoeTensorDescC), c_int32, c_void_p]),
    "moe_plan_weight_bytes": (c_uint64, [c_void_p]),
    "moe_workspace_bytes": (c_uint64, [c_void_p, c_int32]),
    "moe_forward": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_uint64, c_void_p]),
    "moe_forward_timed": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_uint64,
                                    POINTER(c_float), c_void_p]),
    "moe_forward_static_scratch": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p]),
    "moe_route": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                            c_void_p, c_uint64, c_void_p]),
    "moe_ep_dispatch": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_uint64, c_void_p]),
    "moe_ep_workspace_bytes": (c_uint64, [c_void_p, c_int32]),
    "moe_ep_experts": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p,
                                 c_uint64, c_void_p]),
    "moe_ep_shared": (c_int32, [c_void_p, c_int32, c_void_p, c_uint64, c_void_p]),
    "moe_ep_combine": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p,
                                 c_uint64, c_void_p]),
    "moe_ep_capacity": (c_int32, [c_void_p, c_int32]),
    "moe_ep_dispatch_padded": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p,
                                         c_uint64, c_void_p]),
    "moe_ep_padded_workspace_bytes": (c_uint64, [c_void_p, c_int32]),
    "moe_ep_experts_padded": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_uint64,
                                        c_void_p]),
    "moe_ep_token_row_halves": (c_int32, [c_void_p]),
    "moe_ep_token_pack": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p,
                                    c_uint64, c_void_p]),
    "moe_ep_gathered_workspace_bytes": (c_uint64, [c_void_p, c_int32]),
    "moe_ep_experts_gathered": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p,
                                          c_uint64, c_void_p]),
    "moe_ep_combine_partial": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p,
                                         c_void_p, c_uint64, c_void_p]),
    "moe_ep_p2p_pack": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p,
                                  c_void_p, c_int32, c_void_p, c_void_p, c_uint64, c_void_p]),
    "moe_ep_p2p_wait": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int64, c_void_p]),
    "moe_ep_p2p_experts": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p,
                                     c_void_p, c_int32, c_void_p, c_void_p, c_uint64, c_void_p]),
    "moe_ep_p2p_combine": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int32,
                                     c_void_p, c_void_p, c_uint64, c_void_p]),
    "moe_status": (c_int32, [c_void_p, c_void_p]),
    "moe_attn_create": (c_int32, [POINTER(MoeAttnConfigC), POINTER(c_void_p)]),
    "moe_attn_destroy": (c_int32, [c_void_p]),
    "moe_attn_bind": (c_int32, [c_void_p, c_void_p, c_uint64, POINTER(MoeTensorDescC), c_int32,
                                c_void_p]),
    "moe_attn_weight_bytes": (c_uint64, [c_void_p]),
    "moe_attn_workspace_bytes": (c_uint64, [c_void_p, c_int32]),
    "moe_attn_forward": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_uint64,
                                   c_void_p]),
    "moe_attn_status": (c_int32, [c_void_p, c_void_p]),
    "moe_wait_probe": (c_int32, [c_void_p, c_int64, c_void_p]),
    "moe_last_error": (c_char_p, []),
    "moe_version": (c_char_p, []),
    "moe_rt_device_count": (c_int32, [POINTER(c_int32)]),
    "moe_rt_set_device": (c_int32, [c_int32]),
    "moe_rt_can_access_peer": (c_int32, [c_int32, c_int32, POINTER(c_int32)]),
    "moe_rt_malloc": (c_int32, [c_uint64, POINTER(c_void_p)]),
    "moe_rt_free": (c_int32, [c_void_p]),
    "moe_rt_ipc_get_handle": (c_int32, [c_void_p, c_void_p]),
    "moe_rt_ipc_open_handle": (c_int32, [c_void_p, c_void_p]),
    "moe_rt_ipc_close_handle": (c_int32, [c_void_p]),
    "moe_rt_malloc_host": (c_int32, [c_uint64, POINTER(c_void_p)]),
    "moe_rt_free_host": (c_int32, [c_void_p]),
    "moe_rt_stream_create": (c_int32, [POINTER(c_void_p)]),
    "moe_rt_stream_destroy": (c_int32, [c_void_p]),
    "moe_rt_memcpy_h2d_async": (c_int32, [c_void_p, c_void_p, c_uint64, c_void_p]),
    "moe_rt_memcpy_d2h_async": (c_int32, [c_void_p, c_void_p, c_uint64, c_void_p]),
    "moe_rt_memcpy_d2d_async": (c_int32, [c_void_p, c_void_p, c_uint64, c_void_p]),
    "moe_rt_event_record": (c_int32, [c_void_p, POINTER(c_void_p)]),
    "moe_rt_event_destroy": (c_int32, [c_void_p]),
    "moe_rt_stream_wait_event": (c_int32, [c_void_p, c_void_p]),
    "moe_rt_stream_synchronize": (c_int32, [c_void_p]),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load libmoe_sm100.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libmoe_sm100.so not found at {LIB_PATH}: build it with "
                "`python -m moe_sm100.build` (or __graft_entry__.build())")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _PROTOTYPES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int) -> None:
    if rc == MOE_OK:
        return
    msg = lib().moe_last_error().decode(errors="replace")
    if rc in (MOE_ERR_INVALID, MOE_ERR_WORKSPACE):
        raise MoeValueError(rc, msg)
    if rc == MOE_ERR_MISSING_TENSOR:
        raise MoeKeyError(rc, msg)
    raise MoeError(rc, msg)
