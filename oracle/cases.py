"""Seeded synthetic MoE-layer cases for parity tests and the CPU baseline.

TEST INFRASTRUCTURE ONLY (see oracle/moe_oracle.py).  A case is a dict of fp32
numpy arrays named exactly like the reference loader's layer tensors
(offload_runtime/loader/huggingface.py:492-506, 560-575), plus the activations
``x`` and an ``OracleConfig``.  The reference executor consumes the fp32 tensors
unchanged; the CUDA path consumes the same values packed as f16 (bf16-valued
weights) or per-channel INT8.

Distributions follow the benchmark configs: x ~ N(0,1), weights ~ N(0, 0.02),
e_score_correction_bias ~ N(0, 0.01), optional Zipf(s)-ranked bias skew (rank r
gets ``zipf_amp / r**s``, ranks assigned to a seeded permutation of experts).
"""
from __future__ import annotations

from dataclasses import dataclass, asdict
from typing import Any

import numpy as np

from .moe_oracle import OracleConfig, bf16_round, int8_pc_dequantize, int8_pc_quantize


@dataclass
class CaseSpec:
    hidden: int
    n_experts: int
    top_k: int
    inter: int
    shared_inter: int
    tokens: int
    seed: int = 0
    family: str = "glm"            # "glm" (shared_experts., bias) | "qwen3" (shared_expert., gate)
    score_func: str = "softmax"
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 1.0
    eps: float = 1e-5
    weights: str = "bf16"          # "f32" | "bf16" | "int8_pc"
    bias_std: float = 0.01
    zipf_s: float = 0.0            # 0 -> no skew
    zipf_amp: float = 1.0
    norm_w_std: float = 0.0        # 0 -> post_attention_layernorm.weight = 1

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def oracle_config(spec: CaseSpec) -> OracleConfig:
    glm = spec.family == "glm"
    return OracleConfig(
        hidden=spec.hidden, n_experts=spec.n_experts, top_k=spec.top_k, inter=spec.inter,
        shared_inter=spec.shared_inter, score_func=spec.score_func, use_bias=glm,
        norm_topk_prob=spec.norm_topk_prob, routed_scaling_factor=spec.routed_scaling_factor,
        eps=spec.eps, shared_prefix="mlp.shared_experts." if glm else "mlp.shared_expert.",
    )


def _weights(rng: np.random.Generator, shape: tuple[int, int], fmt: str
             ) -> tuple[np.ndarray, tuple[np.ndarray, np.ndarray] | None]:
    w = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02))
    if fmt == "f32":
        return w, None
    if fmt == "bf16":
        return bf16_round(w), None
    if fmt == "int8_pc":
        q, s = int8_pc_quantize(w)
        return int8_pc_dequantize(q, s), (q, s)
    raise ValueError(fmt)


def make_case(spec: CaseSpec) -> tuple[np.ndarray, dict[str, np.ndarray], dict[str, Any], OracleConfig]:
    """Build ``(x, tensors, quant, cfg)``.

    ``tensors`` holds the fp32 values the reference sees; ``quant`` maps expert weight
    names to their ``(int8 q, fp16 scale)`` pair when ``spec.weights == "int8_pc"``.
    """
    rng = np.random.default_rng(spec.seed)
    H, E, I, SI = spec.hidden, spec.n_experts, spec.inter, spec.shared_inter
    x = rng.standard_normal((spec.tokens, H), dtype=np.float32)
    t: dict[str, np.ndarray] = {}
    quant: dict[str, Any] = {}
    if spec.norm_w_std > 0:
        t["post_attention_layernorm.weight"] = (
            1.0 + spec.norm_w_std * rng.standard_normal(H, dtype=np.float32)).astype(np.float32)
    else:
        t["post_attention_layernorm.weight"] = np.ones(H, dtype=np.float32)
    t["mlp.gate.weight"] = rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02)
    if spec.family == "glm":
        bias = rng.standard_normal(E, dtype=np.float32) * np.float32(spec.bias_std)
        if spec.zipf_s > 0:
            ranks = np.arange(1, E + 1, dtype=np.float64)
            skew = (spec.zipf_amp / ranks ** spec.zipf_s).astype(np.float32)
            bias = bias + skew[rng.permutation(E)]
        t["mlp.gate.e_score_correction_bias"] = bias.astype(np.float32)
    for e in range(E):
        for nm, shp in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
            key = f"mlp.experts.{e}.{nm}.weight"
            t[key], qs = _weights(rng, shp, spec.weights)
            if qs is not None:
                quant[key] = qs
    if SI > 0:
        prefix = "mlp.shared_experts." if spec.family == "glm" else "mlp.shared_expert."
        for nm, shp in (("gate_proj", (SI, H)), ("up_proj", (SI, H)), ("down_proj", (H, SI))):
            key = f"{prefix}{nm}.weight"
            t[key], qs = _weights(rng, shp, spec.weights)
            if qs is not None:
                quant[key] = qs
        if spec.family == "qwen3":
            t["mlp.shared_expert_gate.weight"] = (
                rng.standard_normal((1, H), dtype=np.float32) * np.float32(0.02))
    return x, t, quant, oracle_config(spec)


def input_checksum(x: np.ndarray, t: dict[str, np.ndarray]) -> np.ndarray:
    """float64 sums of x and of every tensor (sorted by name): detects RNG drift."""
    vals = [float(np.sum(x, dtype=np.float64))]
    vals += [float(np.sum(t[k], dtype=np.float64)) for k in sorted(t)]
    return np.asarray(vals, dtype=np.float64)


# Fixture cases.  Sizes keep every oracle run to well under a second.
GOLDEN_SPECS: dict[str, CaseSpec] = {
    # BASELINE config 0 (tiny GLM4-MoE style), reference softmax-biased routing
    "glm_cfg0": CaseSpec(hidden=1024, n_experts=16, top_k=4, inter=256, shared_inter=256,
                         tokens=64, seed=0, routed_scaling_factor=2.5, weights="f32"),
    # same shape, per-channel INT8 expert weights, non-trivial norm weight
    "glm_cfg0_int8": CaseSpec(hidden=1024, n_experts=16, top_k=4, inter=256, shared_inter=256,
                              tokens=64, seed=1, routed_scaling_factor=2.5, weights="int8_pc",
                              norm_w_std=0.1),
    # Zipf-skewed routing (uneven expert loads), bf16-valued weights
    "glm_zipf": CaseSpec(hidden=512, n_experts=32, top_k=8, inter=128, shared_inter=128,
                         tokens=96, seed=2, routed_scaling_factor=2.5, zipf_s=1.1),
    # Qwen3-Next style: softmax top-10, no bias, sigmoid-gated shared expert
    "qwen3_small": CaseSpec(hidden=512, n_experts=64, top_k=10, inter=128, shared_inter=128,
                            tokens=33, seed=3, family="qwen3", eps=1e-6, norm_w_std=0.1),
    # ragged / edge token counts, no shared expert, shared intermediate != inter
    "glm_t1_noshared": CaseSpec(hidden=256, n_experts=8, top_k=2, inter=64, shared_inter=0,
                                tokens=1, seed=4, routed_scaling_factor=2.5),
    "glm_t3_si": CaseSpec(hidden=256, n_experts=8, top_k=2, inter=64, shared_inter=96,
                          tokens=3, seed=5, routed_scaling_factor=1.0, norm_w_std=0.1),
    # norm_topk_prob = False
    "glm_nonorm": CaseSpec(hidden=256, n_experts=16, top_k=3, inter=64, shared_inter=64,
                           tokens=17, seed=6, norm_topk_prob=False, routed_scaling_factor=2.5),
}

# HF GLM-4.x sigmoid routing (no reference counterpart; pinned against transformers)
SIGMOID_SPECS: dict[str, CaseSpec] = {
    "glm_sigmoid": CaseSpec(hidden=1024, n_experts=16, top_k=4, inter=256, shared_inter=256,
                            tokens=64, seed=7, score_func="sigmoid", routed_scaling_factor=2.5),
}


# Dense MLP of GLM-4 first_k_dense_replace layers (glm4_moe.py:166-172): only
# hidden, inter (the layer's intermediate_size), tokens, seed, eps and weights
# matter; n_experts / top_k are 0.
DENSE_SPECS: dict[str, CaseSpec] = {
    "glm_dense": CaseSpec(hidden=1024, n_experts=0, top_k=0, inter=512, shared_inter=0,
                          tokens=24, seed=31, weights="bf16", norm_w_std=0.1),
    "glm_dense_t1": CaseSpec(hidden=512, n_experts=0, top_k=0, inter=384, shared_inter=0,
                             tokens=1, seed=32, weights="f32", norm_w_std=0.1),
}


def make_dense_case(spec: CaseSpec) -> tuple[np.ndarray, dict[str, np.ndarray], dict[str, Any]]:
    """``(x, tensors, quant)`` of a dense-MLP layer: post_attention_layernorm and
    mlp.{gate,up,down}_proj (nn.Linear [out, in] layout)."""
    rng = np.random.default_rng(spec.seed)
    H, I = spec.hidden, spec.inter
    x = rng.standard_normal((spec.tokens, H), dtype=np.float32)
    t: dict[str, np.ndarray] = {}
    quant: dict[str, Any] = {}
    t["post_attention_layernorm.weight"] = (
        1.0 + spec.norm_w_std * rng.standard_normal(H, dtype=np.float32)).astype(np.float32)
    for nm, shp in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
        key = f"mlp.{nm}.weight"
        t[key], qs = _weights(rng, shp, spec.weights)
        if qs is not None:
            quant[key] = qs
    return x, t, quant


# ---------------------------------------------------------------------------
# GLM-4 MoE attention blocks (glm4_moe.py:112-162)
# ---------------------------------------------------------------------------
@dataclass
class AttnSpec:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    tokens: int
    seed: int = 0
    qk_norm: bool = True
    bias: bool = True
    partial_rotary_factor: float = 0.5
    rope_theta: float = 1_000_000.0
    eps: float = 1e-5
    weights: str = "bf16"          # "f32" | "bf16"
    norm_w_std: float = 0.1

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    def hf_config(self) -> dict[str, Any]:
        """The config keys GLM4MoeExecutor reads for its attention (glm4_moe.py:70-84)."""
        return {"hidden_size": self.hidden, "num_attention_heads": self.heads,
                "num_key_value_heads": self.kv_heads, "head_dim": self.head_dim,
                "rms_norm_eps": self.eps, "rope_theta": self.rope_theta,
                "partial_rotary_factor": self.partial_rotary_factor,
                "intermediate_size": 4 * self.hidden}


def make_attn_tensors(spec: AttnSpec, rng: np.random.Generator) -> dict[str, np.ndarray]:
    """Attention tensors of one layer, named as the loader names them
    (``input_layernorm.weight``, ``self_attn.{q,k,v,o}_proj.weight``, biases,
    ``self_attn.{q,k}_norm.weight``)."""
    H, nh, nkv, hd = spec.hidden, spec.heads, spec.kv_heads, spec.head_dim
    t: dict[str, np.ndarray] = {}
    t["input_layernorm.weight"] = (
        1.0 + spec.norm_w_std * rng.standard_normal(H, dtype=np.float32)).astype(np.float32)
    for name, rows in (("q", nh * hd), ("k", nkv * hd), ("v", nkv * hd)):
        t[f"self_attn.{name}_proj.weight"], _ = _weights(rng, (rows, H), spec.weights)
        if spec.bias:
            t[f"self_attn.{name}_proj.bias"] = (
                rng.standard_normal(rows, dtype=np.float32) * np.float32(0.02))
    if spec.qk_norm:
        for name in ("q", "k"):
            t[f"self_attn.{name}_norm.weight"] = (
                1.0 + spec.norm_w_std * rng.standard_normal(hd, dtype=np.float32)).astype(np.float32)
    t["self_attn.o_proj.weight"], _ = _weights(rng, (H, nh * hd), spec.weights)
    return t


def make_attn_case(spec: AttnSpec) -> tuple[np.ndarray, dict[str, np.ndarray]]:
    rng = np.random.default_rng(spec.seed)
    x = rng.standard_normal((spec.tokens, spec.hidden), dtype=np.float32)
    return x, make_attn_tensors(spec, rng)


ATTN_SPECS: dict[str, AttnSpec] = {
    # GLM-4.5/4.7 style: GQA, per-head q/k norm, q/k/v bias, half the head rotated
    "attn_glm_small": AttnSpec(hidden=256, heads=4, kv_heads=2, head_dim=64, tokens=17, seed=41),
    # full rotary embedding, no q/k norm, no bias, plain multi-head
    "attn_glm_fullrope": AttnSpec(hidden=256, heads=4, kv_heads=4, head_dim=64, tokens=5, seed=42,
                                  qk_norm=False, bias=False, partial_rotary_factor=1.0,
                                  rope_theta=10000.0, weights="f32"),
    # a single token (the first decode step of a fresh sequence)
    "attn_glm_t1": AttnSpec(hidden=256, heads=4, kv_heads=1, head_dim=64, tokens=1, seed=43),
    # GLM-4.7 head geometry (head_dim 128, 8 query heads per kv head), two key tiles
    "attn_glm_mid": AttnSpec(hidden=1024, heads=16, kv_heads=2, head_dim=128, tokens=200, seed=44),
}
