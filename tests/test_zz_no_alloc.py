"""The allocation-free forward, ``moe_forward_static_scratch`` (needs a B200).

Some callers of this library only own the buffers they hand in: a Go / Java / C
host behind a thin FFI that holds just the activations, a process whose memory
pool has already taken the GPU, or a serving loop that may not call cudaMalloc
because it synchronises the device.  For them the library runs the MoE forward
with a fixed scratch array of its own instead of a caller workspace.

These tests call that entry point through the C ABI and compare its output with
``moe_forward`` (the workspace entry point) on calls in a row, with different
batches so that each call runs over the previous call's leftovers.  Both paths
launch the same deterministic kernels on the same weights and inputs, so the
outputs must be identical bit for bit: any difference means leftover scratch
contents leaked into a result.  Covered: decode batches (one-CTA routing tail),
a prefill batch (T > 256: tensor-core router, permutation counters), a dense-MLP
plan, the refusal of a batch too large for the fixed scratch, and that the
caller's current device is left alone.  The file is named so that pytest
collects it last.
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


def _dense_layer(max_tokens: int) -> MoeLayer:
    rng = np.random.default_rng(78)
    inter = 384
    t = {"post_attention_layernorm.weight": (1 + 0.1 * rng.standard_normal(H)).astype(np.float32),
         "mlp.gate_proj.weight": (rng.standard_normal((inter, H)) * 0.02).astype(np.float32),
         "mlp.up_proj.weight": (rng.standard_normal((inter, H)) * 0.02).astype(np.float32),
         "mlp.down_proj.weight": (rng.standard_normal((H, inter)) * 0.02).astype(np.float32)}
    blob, meta = pack_layer(t, expert_format="bfloat16")
    ml = MoeLayer(MoeLayerConfig.dense_mlp({"hidden_size": H, "intermediate_size": inter},
                                           rms_norm_eps=1e-5, max_tokens=max_tokens))
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


def _assert_same(got: "torch.Tensor", ref: "torch.Tensor", what: str) -> None:
    # identical kernels on identical inputs: any difference is leftover scratch
    assert torch.equal(got, ref), f"{what}: differs from moe_forward (rel-L2 {_rel_l2(got, ref):.3e})"


def test_static_scratch_matches_workspace_forward_twice() -> None:
    ml = _layer(max_tokens=384)
    gen = torch.Generator(device="cuda").manual_seed(5)
    batches = [torch.randn((t, H), generator=gen, device="cuda") for t in (96, 7, 300, 13)]
    refs = [_forward_workspace(ml, x) for x in batches]
    device_before = torch.cuda.current_device()
    # the first call on this device sets up the scratch address; each later call
    # runs over the scratch the previous one left (decode, decode, prefill, decode)
    gots = [_forward_static(ml, x) for x in batches]
    torch.cuda.synchronize()
    ml.status()
    assert torch.cuda.current_device() == device_before
    for i, (got, ref) in enumerate(zip(gots, refs)):
        _assert_same(got, ref, f"call {i + 1} (T={batches[i].shape[0]})")
    ml.close()


def test_static_scratch_dense_plan() -> None:
    ml = _dense_layer(max_tokens=64)
    gen = torch.Generator(device="cuda").manual_seed(6)
    xs = [torch.randn((t, H), generator=gen, device="cuda") for t in (40, 3)]
    refs = [_forward_workspace(ml, x) for x in xs]
    gots = [_forward_static(ml, x) for x in xs]
    torch.cuda.synchronize()
    ml.status()
    for i, (got, ref) in enumerate(zip(gots, refs)):
        _assert_same(got, ref, f"dense call {i + 1}")
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
