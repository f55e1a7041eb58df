"""Host-side logic of moe_sm100 that needs no GPU: packing, formats, config parsing,
dequantizers (mirroring the reference's tests/test_quantize.py known answers),
residency pool and executor guards."""
from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

from moe_sm100.buffer_pool import ResidentLayerPool
from moe_sm100.config import MoeLayerConfig
from moe_sm100.layer import _descs, layer_shapes
from moe_sm100.packing import (bf16_bits, bf16_to_f32, dequantize_int8_per_channel, is_expert_weight,
                               pack_layer, quantize_int8_per_channel)
from moe_sm100.quantize import Int8PerChannelDequantizer
from moe_sm100.types import DeviceBuffer, HostBuffer, LayerSpec
from oracle.moe_oracle import bf16_round, int8_pc_quantize


# ------------------------------------------------------------------ formats
def test_bf16_bits_match_torch_rounding() -> None:
    rng = np.random.default_rng(0)
    a = (rng.standard_normal(10000) * 10.0 ** rng.integers(-8, 8, 10000)).astype(np.float32)
    a[:4] = [0.0, -0.0, np.inf, -np.inf]
    ours = bf16_bits(a)
    ref = torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, ref)
    np.testing.assert_array_equal(bf16_to_f32(ours), bf16_round(a))


def test_int8_quantizer_matches_oracle_format() -> None:
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((64, 96)) * 0.02).astype(np.float32)
    w[3] = 0.0
    q, s = quantize_int8_per_channel(w)
    q2, s2 = int8_pc_quantize(w)
    np.testing.assert_array_equal(q, q2)
    np.testing.assert_array_equal(s.view(np.uint16), s2.view(np.uint16))
    assert np.all(q[3] == 0) and s[3] == 0
    assert np.abs(q).max() == 127
    err = np.abs(dequantize_int8_per_channel(q, s) - w)
    assert np.all(err <= s.astype(np.float32)[:, None] * 0.5 + 1e-6)


def test_expert_weight_names() -> None:
    assert is_expert_weight("mlp.experts.12.gate_proj.weight")
    assert is_expert_weight("model.layers.3.mlp.experts.0.down_proj.weight")
    assert is_expert_weight("mlp.shared_experts.up_proj.weight")
    assert is_expert_weight("mlp.shared_expert.down_proj.weight")
    assert not is_expert_weight("mlp.gate.weight")
    assert not is_expert_weight("mlp.shared_expert_gate.weight")
    assert not is_expert_weight("self_attn.q_proj.weight")
    # dense MLP of first_k_dense_replace layers: packed like expert weights
    assert is_expert_weight("mlp.gate_proj.weight")
    assert is_expert_weight("model.layers.0.mlp.down_proj.weight")
    assert not is_expert_weight("mlp.gate_proj.bias")


@pytest.mark.parametrize("fmt", ["float32", "bfloat16", "int8"])
def test_pack_layer_roundtrip(fmt: str) -> None:
    rng = np.random.default_rng(2)
    t = {
        "post_attention_layernorm.weight": np.ones(32, np.float32),
        "mlp.gate.weight": rng.standard_normal((4, 32)).astype(np.float32),
        "mlp.experts.0.gate_proj.weight": (rng.standard_normal((16, 32)) * 0.02).astype(np.float32),
        "mlp.experts.0.down_proj.weight": (rng.standard_normal((32, 16)) * 0.02).astype(np.float32),
    }
    blob, meta = pack_layer(t, expert_format=fmt)
    names = [m["name"] for m in meta]
    assert names == sorted(names)  # loader order (huggingface.py:492-506)
    by = {m["name"]: m for m in meta}
    for m in meta:
        assert m["offset"] % 256 == 0
    router = np.frombuffer(blob, np.float32, count=4 * 32, offset=by["mlp.gate.weight"]["offset"])
    np.testing.assert_array_equal(router.reshape(4, 32), t["mlp.gate.weight"])
    m = by["mlp.experts.0.gate_proj.weight"]
    assert m["dtype"] == {"float32": "float32", "bfloat16": "bfloat16", "int8": "int8"}[fmt]
    if fmt == "int8":
        assert "mlp.experts.0.gate_proj.weight_scale" in by
        s = by["mlp.experts.0.gate_proj.weight_scale"]
        assert s["dtype"] == "float16" and s["shape"] == [16]
    d, keep = _descs(meta)
    assert len(d) == len(meta) and d[0].name == meta[0]["name"].encode()


# ------------------------------------------------------------------ config
def test_glm_config_defaults_follow_reference() -> None:
    c = MoeLayerConfig.glm4_moe({"hidden_size": 5120, "moe_intermediate_size": 1536})
    assert (c.n_experts, c.top_k, c.routed_scaling_factor, c.rms_norm_eps) == (160, 8, 2.5, 1e-5)
    assert c.norm_topk_prob and c.use_bias and not c.has_shared_gate
    assert c.score_func == "softmax"
    s = MoeLayerConfig.glm4_moe({"hidden_size": 8}, score_func="sigmoid")
    assert s.score_func == "sigmoid"
    cc = c.to_c()
    assert cc.hidden == 5120 and cc.n_experts == 160 and abs(cc.routed_scaling_factor - 2.5) < 1e-7


def test_dense_mlp_config() -> None:
    c = MoeLayerConfig.dense_mlp({"hidden_size": 5120, "intermediate_size": 12288,
                                  "rms_norm_eps": 1e-5})
    assert (c.n_experts, c.top_k, c.shared_inter, c.inter) == (0, 0, 12288, 0)
    assert not c.use_bias and not c.has_shared_gate and c.rms_norm_eps == 1e-5
    cc = c.to_c()
    assert cc.n_experts == 0 and cc.shared_inter == 12288


def test_qwen3_config_defaults_follow_reference() -> None:
    c = MoeLayerConfig.qwen3_next({"hidden_size": 2048})
    assert (c.n_experts, c.top_k, c.inter, c.shared_inter) == (512, 10, 512, 512)
    assert c.routed_scaling_factor == 1.0 and not c.use_bias and c.has_shared_gate
    c2 = MoeLayerConfig.qwen3_next({"hidden_size": 64, "n_routed_experts": 32})
    assert c2.n_experts == 32
    with pytest.raises(ValueError):
        MoeLayerConfig.qwen3_next({"hidden_size": 64}, score_func="relu").to_c()


def test_layer_shapes_from_metadata() -> None:
    meta = [{"name": "mlp.experts.0.gate_proj.weight", "shape": [96, 64]},
            {"name": "mlp.shared_expert.gate_proj.weight", "shape": [48, 64]},
            {"name": "mlp.shared_expert_gate.weight", "shape": [1, 64]}]
    assert layer_shapes(meta) == {"inter": 96, "shared_inter": 48, "has_shared_gate": True}


# ------------------------------------------------------------------ dequantizers
def test_per_channel_dequantizer_keeps_blob_compressed_by_default() -> None:
    rng = np.random.default_rng(3)
    t = {"mlp.experts.0.up_proj.weight": (rng.standard_normal((16, 32)) * 0.02).astype(np.float32),
         "mlp.gate.weight": rng.standard_normal((2, 32)).astype(np.float32)}
    blob, meta = pack_layer(t, expert_format="int8")
    layer = LayerSpec(0, "L0", len(blob), {"dtype": "int8_per_channel", "tensors": meta})
    keep = Int8PerChannelDequantizer()
    assert not keep.needs_dequantize(layer)
    assert keep.decompressed_nbytes(layer) == layer.nbytes
    host = Int8PerChannelDequantizer(keep_on_device=False)
    assert host.needs_dequantize(layer)
    out = host.dequantize(layer, HostBuffer(memoryview(blob)))
    om = {m["name"]: m for m in layer.metadata["dequantized_tensors"]}
    m = om["mlp.experts.0.up_proj.weight"]
    w = np.frombuffer(out.view, np.float32, count=16 * 32, offset=m["offset"]).reshape(16, 32)
    q, s = quantize_int8_per_channel(t["mlp.experts.0.up_proj.weight"])
    np.testing.assert_array_equal(w, dequantize_int8_per_channel(q, s))


# ------------------------------------------------------------------ residency
def test_resident_pool_budget_and_lru_eviction() -> None:
    released: list[int] = []
    evicted: list[int] = []
    pool = ResidentLayerPool(budget_bytes=100, on_evict=evicted.append)
    for lid in range(3):
        assert pool.admit(lid, 40, lambda lid=lid: released.append(lid))
    assert evicted == [0] and released == [0] and pool.resident_bytes == 80
    assert pool.touch(1)  # 2 is now the oldest
    assert pool.admit(3, 40, lambda: released.append(3))
    assert evicted == [0, 2] and 1 in pool and pool.is_resident(3)
    # a layer larger than the whole budget is refused without releasing anything
    assert not pool.admit(9, 101, lambda: released.append(9))
    assert released == [0, 2] and not pool.touch(9)
    # admitting a resident layer again replaces (and releases) the old entry
    assert pool.admit(3, 10, lambda: released.append(33))
    assert released == [0, 2, 3] and pool.resident_bytes == 50
    pool.drain()
    assert sorted(released) == [0, 1, 2, 3, 33] and pool.resident_bytes == 0


def test_executor_rejects_non_cuda_backend() -> None:
    from moe_sm100.executors import GLM4MoeExecutor
    ex = GLM4MoeExecutor({"hidden_size": 256, "moe_intermediate_size": 64, "n_routed_experts": 8,
                          "num_experts_per_tok": 2})
    assert ex.num_experts_per_tok == 2 and ex.routed_scaling_factor == 2.5
    layer = LayerSpec(1, "model.layers.1", 0, {"tensors": [], "is_moe": True})

    class _Null:
        name = "null"

    with pytest.raises(ValueError):
        ex.run_layer(layer, np.zeros((1, 256), np.float32), DeviceBuffer(0, 0, "null"), _Null(), None)


def test_synthetic_expert_subsets_agree_across_ranks() -> None:
    """An expert-parallel rank builds only its experts; the router, bias and shared
    expert, and every expert two ranks both hold, come out the same."""
    from moe_sm100.synthetic import SyntheticSpec, build_device_layer, host_tensor
    kw = dict(hidden=64, n_experts=8, top_k=2, inter=32, shared_inter=32, family="glm",
              expert_dtype="int8", seed=5, zipf_s=1.1)
    b1, m1 = build_device_layer(SyntheticSpec(**kw, experts=(0, 4)), device="cpu")
    b2, m2 = build_device_layer(SyntheticSpec(**kw, experts=(2, 6)), device="cpu")
    experts1 = {m["name"].split(".")[2] for m in m1 if m["name"].startswith("mlp.experts.")}
    assert experts1 == {"0", "1", "2", "3"}
    for name in ("mlp.gate.weight", "mlp.gate.e_score_correction_bias",
                 "mlp.experts.2.up_proj.weight", "mlp.experts.3.down_proj.weight_scale",
                 "mlp.shared_experts.gate_proj.weight"):
        np.testing.assert_array_equal(host_tensor(b1, m1, name), host_tensor(b2, m2, name))
    with pytest.raises(ValueError, match="outside"):
        build_device_layer(SyntheticSpec(**kw, experts=(4, 9)), device="cpu")


def test_stack_bench_memory_plan() -> None:
    """The 89-layer INT8 stack's resident bytes per GPU (bench.py --stack decides
    from this whether a world size fits before building anything)."""
    import importlib.util
    import os
    spec = importlib.util.spec_from_file_location(
        "bench_mod", os.path.join(os.path.dirname(os.path.dirname(__file__)), "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    gib = [bench._stack_resident_bytes(160 // n, 89) / 2**30 for n in (2, 4, 8)]
    # 160/N experts x 3 x 5120 x 1536 int8 + row scales + shared expert + router, per layer
    assert 158 < gib[0] < 160 and 80 < gib[1] < 81.5 and 41 < gib[2] < 42
    # the expert share halves with each doubling; router and shared expert stay
    assert abs((gib[0] - gib[1]) - 2 * (gib[1] - gib[2])) < 0.01


def test_prefill_gemm_roofline_bytes() -> None:
    """bench.py's prefill GEMM floors: the touched experts' weights once, the token rows
    in and the activations / outputs out.  With ~160 tokens per expert and 16-bit
    weights (the Qwen3-Next prefill) the weight stream, not the tensor work, bounds the
    GEMMs; the GLM-4.7 INT8 prefill (~205 tokens per expert, 1-byte weights) is
    tensor-bound."""
    import importlib.util
    import os
    spec = importlib.util.spec_from_file_location(
        "bench_mod", os.path.join(os.path.dirname(os.path.dirname(__file__)), "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    T, k, H, I, SI = 8192, 10, 2048, 512, 512
    bg, bd = bench._gemm_bytes(T, k, H, I, SI, 512, 2)
    w_gu, w_d = (512 * 2 * I * H + 2 * SI * H) * 2, (512 * H * I + H * SI) * 2
    rows = T * k
    assert bg == w_gu + (rows + T) * H * 2 + (rows * I + T * SI) * 2
    assert bd == w_d + (rows * I + T * SI) * 2 + rows * H * 2 + T * H * 4
    fg, fd = bench._gemm_flops(T, k, H, I, SI)
    tc, hbm = 1666.7e12, 6536e9  # the measured peaks of this pool's B200s
    assert bg / hbm > fg / tc and bd / hbm > fd / tc      # Qwen3 prefill: weight-bound
    fg8, _ = bench._gemm_flops(4096, 8, 5120, 1536, 1536)
    bg8, _ = bench._gemm_bytes(4096, 8, 5120, 1536, 1536, 160, 1)
    assert fg8 / tc > bg8 / hbm                           # GLM INT8 prefill: tensor-bound
    # no shared expert: no shared rows or shared weights
    bg0, bd0 = bench._gemm_bytes(64, 8, 1024, 256, 0, 16, 2)
    assert bg0 == 16 * 2 * 256 * 1024 * 2 + 64 * 8 * 1024 * 2 + 64 * 8 * 256 * 2
    assert bd0 == 16 * 1024 * 256 * 2 + 64 * 8 * 256 * 2 + 64 * 8 * 1024 * 2


def test_fixed_capacity_needs_a_capacity() -> None:
    from moe_sm100.ep import ExpertParallelMoe

    class NoCapacity:
        def capacity(self, tokens: int) -> int:
            return 0

    with pytest.raises(ValueError, match="capacity"):
        ExpertParallelMoe(NoCapacity(), padded_tokens=8)
    ExpertParallelMoe(NoCapacity(), padded_tokens=0)  # exact exchange only: no capacity asked


def test_tensor_dict_cache_never_serves_other_weights() -> None:
    """``_moe_mlp_block(x, t)`` with host dicts: a dict is matched by the arrays it
    holds, not by its id (which CPython reuses), and the cache stays bounded."""
    from moe_sm100.executors import GLM4MoeExecutor

    class _FakeLayer:
        def __init__(self, tag: int) -> None:
            self.tag, self.closed = tag, False

        def close(self) -> None:
            self.closed = True

    ex = GLM4MoeExecutor({"hidden_size": 64, "moe_intermediate_size": 16, "n_routed_experts": 4,
                          "num_experts_per_tok": 2})
    made: list[_FakeLayer] = []

    def fake_bind(t, expert_format="float32", dense=False):  # noqa: ANN001, ANN202
        made.append(_FakeLayer(len(made)))
        return made[-1]

    ex.bind_tensors = fake_bind  # type: ignore[method-assign]
    t1 = {"mlp.gate.weight": np.zeros((4, 64), np.float32)}
    a = ex._layer_for_tensors(t1, dense=False)
    assert ex._layer_for_tensors(t1, dense=False) is a  # same dict, same arrays: hit
    t1["mlp.gate.weight"] = np.ones((4, 64), np.float32)  # same dict id, new array
    b = ex._layer_for_tensors(t1, dense=False)
    assert b is not a and a.closed
    keep = [{"mlp.gate.weight": np.zeros((4, 64), np.float32)} for _ in range(2)]
    for t in keep:
        ex._layer_for_tensors(t, dense=False)
    assert len(ex._by_tensors) == ex.tensor_cache_size and b.closed
    # a collected dict whose id comes back with other arrays is not a hit
    for _ in range(3):
        c = ex._layer_for_tensors({"mlp.gate.weight": np.zeros((4, 64), np.float32)}, dense=False)
        assert c is made[-1]
