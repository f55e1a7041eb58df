"""The allocation-free forward, ``moe_forward_static_scratch`` (needs a B200).

Some callers of this library only own the buffers they hand in: a Go / Java / C
host behind a thin FFI that holds just the activations, a process whose memory
pool has already taken the GPU, or a serving loop that may not call cudaMalloc
because it synchronises the device.  For them the library runs the MoE forward
with a fixed scratch array of its own instead of a caller workspace.

This test calls that entry point through the C ABI and checks its output
against ``moe_forward`` (the workspace entry point) on two calls in a row, with
different batches so the second call runs over the first call's leftovers, and
checks that a batch too large for the fixed scratch is refused with a clear
error.  It lives in its own file so that pytest collects it last.
"""
from __future__ import annotations

from ctypes import c_void_p

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

from moe_sm100 import MoeLayer, MoeLayerConfig, _lib  # noqa: E402
from moe_sm100.packing import pack_layer  # noqa: E402

TOL = 2e-3  # the rel-L2 bound the 16-bit parity tests use
H, E, K, I, SI = 512, 32, 8, 128, 128


def _layer(max_tokens: int) -> MoeLayer:
    rng = np.random.default_rng(77)
    t = {"post_attention_layernorm.weight": (1 + 0.1 * rng.standard_normal(H)).astype(np.float32),
         "mlp.gate.weight": (rng.standard_normal((E, H)) * 0.02).astype(np.float32),
         "mlp.gate.e_score_correction_bias": (rng.standard_normal(E) * 0.01).astype(np.float32)}
    for e in range(E):
        t[f"mlp.experts.{e}.gate_proj.weight"] = (rng.standard_normal((I, H)) * 0.02).astype(np.float32)
        t[f"mlp.experts.{e}.up_proj.weight"] = (rng.standard_normal((I, H)) * 0.02).astype(np.float32)
        t[f"mlp.experts.{e}.down_proj.weight"] = (rng.standard_normal((H, I)) * 0.02).astype(np.float32)
    t["mlp.shared_experts.gate_proj.weight"] = (rng.standard_normal((SI, H)) * 0.02).astype(np.float32)
    t["mlp.shared_experts.up_proj.weight"] = (rng.standard_normal((SI, H)) * 0.02).astype(np.float32)
    t["mlp.shared_experts.down_proj.weight"] = (rng.standard_normal((H, SI)) * 0.02).astype(np.float32)
    blob, meta = pack_layer(t, expert_format="bfloat16")
    ml = MoeLayer(MoeLayerConfig(hidden=H, n_experts=E, top_k=K, inter=I, shared_inter=SI,
                                 routed_scaling_factor=2.5, rms_norm_eps=1e-5,
                                 max_tokens=max_tokens))
    ml.bind_host(blob, meta)
    return ml


def _forward_workspace(ml: MoeLayer, x: "torch.Tensor") -> "torch.Tensor":
    out = torch.empty_like(x)
    nbytes = int(_lib.lib().moe_workspace_bytes(ml._plan, x.shape[0]))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().moe_forward(ml._plan, c_void_p(x.data_ptr()), c_void_p(out.data_ptr()),
                                      x.shape[0], c_void_p(ws.data_ptr()), nbytes,
                                      c_void_p(stream)))
    return out


def _forward_static(ml: MoeLayer, x: "torch.Tensor") -> "torch.Tensor":
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().moe_forward_static_scratch(
        ml._plan, c_void_p(x.data_ptr()), c_void_p(out.data_ptr()), x.shape[0], c_void_p(stream)))
    return out


def _rel_l2(a: "torch.Tensor", b: "torch.Tensor") -> float:
    a64, b64 = a.double(), b.double()
    return float((a64 - b64).norm() / b64.norm())


def test_static_scratch_matches_workspace_forward_twice() -> None:
    ml = _layer(max_tokens=128)
    gen = torch.Generator(device="cuda").manual_seed(5)
    x1 = torch.randn((96, H), generator=gen, device="cuda")
    x2 = torch.randn((7, H), generator=gen, device="cuda")
    ref1 = _forward_workspace(ml, x1)
    ref2 = _forward_workspace(ml, x2)
    got1 = _forward_static(ml, x1)   # first call on this device sets up the scratch address
    got2 = _forward_static(ml, x2)   # second call reuses the scratch left by the first
    torch.cuda.synchronize()
    ml.status()
    assert _rel_l2(got1, ref1) <= TOL
    assert _rel_l2(got2, ref2) <= TOL
    ml.close()


def test_static_scratch_rejects_batches_beyond_its_size() -> None:
    ml = _layer(max_tokens=4096)
    assert int(_lib.lib().moe_workspace_bytes(ml._plan, 4096)) > _lib.MOE_STATIC_SCRATCH_BYTES
    x = torch.zeros((4096, H), device="cuda")
    out = torch.empty_like(x)
    rc = _lib.lib().moe_forward_static_scratch(ml._plan, c_void_p(x.data_ptr()),
                                               c_void_p(out.data_ptr()), 4096,
                                               c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.MOE_ERR_WORKSPACE
    assert "static scratch" in _lib.lib().moe_last_error().decode()
    ml.close()
