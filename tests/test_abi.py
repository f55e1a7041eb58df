"""The C ABI: the library builds for sm_100a, loads, exports every symbol the header
declares, and rejects bad configurations with status codes (no GPU needed)."""
from __future__ import annotations

import ctypes
import os
import re
from ctypes import byref, c_void_p

import pytest

from moe_sm100 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "moe_sm100.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points() -> None:
    names = declared_functions()
    for required in ("moe_plan_create", "moe_bind_layer", "moe_forward", "moe_route",
                     "moe_workspace_bytes", "moe_last_error", "moe_status"):
        assert required in names


def test_library_exports_every_declared_symbol(built_lib: str) -> None:
    handle = ctypes.CDLL(built_lib)
    missing = [n for n in declared_functions() if not hasattr(handle, n)]
    assert not missing, missing


def test_python_prototypes_cover_header(built_lib: str) -> None:
    assert set(declared_functions()) == set(_lib._PROTOTYPES)


def _cfg(**kw: int) -> _lib.MoeConfigC:
    base = dict(hidden=256, n_experts=8, top_k=2, inter=64, shared_inter=64, score_func=0,
                norm_topk_prob=1, use_bias=1, has_shared_gate=0, weight_format=0,
                routed_scaling_factor=2.5, rms_norm_eps=1e-5, max_tokens=16, expert_begin=0,
                expert_end=0, device=0)
    base.update(kw)
    return _lib.MoeConfigC(**base)


@pytest.mark.parametrize("bad,code", [
    (dict(hidden=100), _lib.MOE_ERR_UNSUPPORTED),
    (dict(inter=40), _lib.MOE_ERR_UNSUPPORTED),
    (dict(top_k=9), _lib.MOE_ERR_INVALID),
    (dict(top_k=0), _lib.MOE_ERR_INVALID),
    (dict(score_func=7), _lib.MOE_ERR_INVALID),
    (dict(weight_format=5), _lib.MOE_ERR_INVALID),
    (dict(max_tokens=0), _lib.MOE_ERR_INVALID),
    (dict(shared_inter=0, has_shared_gate=1), _lib.MOE_ERR_INVALID),
    (dict(n_experts=2000), _lib.MOE_ERR_UNSUPPORTED),
    (dict(n_experts=-1), _lib.MOE_ERR_UNSUPPORTED),
    # dense MLP plans (n_experts = 0): no routing, no bias, a shared width
    (dict(n_experts=0, top_k=2), _lib.MOE_ERR_INVALID),
    (dict(n_experts=0, top_k=0, use_bias=1), _lib.MOE_ERR_INVALID),
    (dict(n_experts=0, top_k=0, use_bias=0, shared_inter=0), _lib.MOE_ERR_INVALID),
    (dict(n_experts=0, top_k=0, use_bias=0, has_shared_gate=1), _lib.MOE_ERR_INVALID),
])
def test_plan_create_validates_before_touching_cuda(built_lib: str, bad: dict, code: int) -> None:
    lib = _lib.lib()
    plan = c_void_p()
    rc = lib.moe_plan_create(byref(_cfg(**bad)), byref(plan))
    assert rc == code
    assert lib.moe_last_error().decode()
    assert not plan.value


def test_null_arguments_are_errors_not_crashes(built_lib: str) -> None:
    lib = _lib.lib()
    assert lib.moe_plan_create(None, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_workspace_bytes(None, 4) == 0
    assert lib.moe_forward(None, None, None, 1, None, 0, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_route(None, None, 1, None, None, None, None, None, 0, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_status(None, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_ep_capacity(None, 5) == 0
    assert lib.moe_ep_padded_workspace_bytes(None, 5) == 0
    assert lib.moe_ep_dispatch_padded(None, None, 1, 8, None, None, 0, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_ep_experts_padded(None, None, 8, None, None, 0, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_plan_destroy(None) == _lib.MOE_OK
    assert b"sm_100a" in lib.moe_version()


def test_check_maps_codes_to_reference_exception_types(built_lib: str) -> None:
    lib = _lib.lib()
    lib.moe_plan_create(None, None)
    with pytest.raises(ValueError):
        _lib.check(_lib.MOE_ERR_INVALID)
    with pytest.raises(KeyError):
        _lib.check(_lib.MOE_ERR_MISSING_TENSOR)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.MOE_ERR_CUDA)
