"""A small GLM-4 MoE checkpoint on disk for the runtime tests (test helper).

Same tensor names and config keys as a Glm4MoeForCausalLM checkpoint (the
reference's own integration fixture, tests/test_integration_inference.py:273-337,
follows the same layout), with the hidden size a multiple of 16 so the device
path accepts it: layer 0 is dense (``first_k_dense_replace = 1``), the others
MoE with a shared expert.  Projection weights are bf16 in the file (their values
are exact in f16), norms / router / biases fp32.

``layer_specs`` describes the layers the way the reference HF loader groups a
GLM-4 MoE checkpoint (offload_runtime/loader/huggingface.py:458-517): short
tensor names, ``full_prefix`` and ``is_moe`` in the metadata.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import numpy as np

from moe_sm100.loader import write_safetensors
from moe_sm100.packing import bf16_bits, bf16_to_f32
from moe_sm100.types import LayerSpec

CONFIG: dict[str, Any] = {
    "architectures": ["Glm4MoeForCausalLM"],
    "hidden_size": 256, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
    "num_hidden_layers": 3, "intermediate_size": 512, "moe_intermediate_size": 64,
    "vocab_size": 64, "rms_norm_eps": 1e-5, "rope_theta": 10000.0,
    "partial_rotary_factor": 0.5, "use_qk_norm": True, "first_k_dense_replace": 1,
    "n_routed_experts": 8, "n_shared_experts": 1, "num_experts_per_tok": 2,
    "routed_scaling_factor": 2.5, "norm_topk_prob": True,
}

_DENSE_ORDER = ["input_layernorm.weight",
                "self_attn.q_proj.weight", "self_attn.q_proj.bias",
                "self_attn.k_proj.weight", "self_attn.k_proj.bias",
                "self_attn.v_proj.weight", "self_attn.v_proj.bias",
                "self_attn.q_norm.weight", "self_attn.k_norm.weight",
                "self_attn.o_proj.weight", "post_attention_layernorm.weight",
                "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"]


def write_model(model_dir: Path, seed: int = 11) -> dict[str, np.ndarray]:
    """Write config.json + model.safetensors; returns every tensor as fp32 values."""
    c = CONFIG
    rng = np.random.default_rng(seed)
    H, nh, nkv, hd = c["hidden_size"], c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
    I, E = c["moe_intermediate_size"], c["n_routed_experts"]
    vals: dict[str, np.ndarray] = {}
    bf: set[str] = set()

    def w(name: str, shape: tuple[int, ...], std: float = 0.02, bf16: bool = True) -> None:
        a = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std))
        if bf16:
            a = bf16_to_f32(bf16_bits(a))
            bf.add(name)
        vals[name] = a

    def norm(name: str, n: int) -> None:
        vals[name] = (1.0 + 0.1 * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)

    w("model.embed_tokens.weight", (c["vocab_size"], H), 1.0, bf16=False)
    norm("model.norm.weight", H)
    w("lm_head.weight", (c["vocab_size"], H), 0.05, bf16=False)
    for layer in range(c["num_hidden_layers"]):
        p = f"model.layers.{layer}."
        norm(p + "input_layernorm.weight", H)
        for n, rows in (("q", nh * hd), ("k", nkv * hd), ("v", nkv * hd)):
            w(f"{p}self_attn.{n}_proj.weight", (rows, H))
            w(f"{p}self_attn.{n}_proj.bias", (rows,), bf16=False)
        norm(p + "self_attn.q_norm.weight", hd)
        norm(p + "self_attn.k_norm.weight", hd)
        w(p + "self_attn.o_proj.weight", (H, nh * hd))
        norm(p + "post_attention_layernorm.weight", H)
        if layer < c["first_k_dense_replace"]:
            inter = c["intermediate_size"]
            w(p + "mlp.gate_proj.weight", (inter, H))
            w(p + "mlp.up_proj.weight", (inter, H))
            w(p + "mlp.down_proj.weight", (H, inter))
            continue
        w(p + "mlp.gate.weight", (E, H), bf16=False)
        w(p + "mlp.gate.e_score_correction_bias", (E,), 0.01, bf16=False)
        for e in range(E):
            w(f"{p}mlp.experts.{e}.gate_proj.weight", (I, H))
            w(f"{p}mlp.experts.{e}.up_proj.weight", (I, H))
            w(f"{p}mlp.experts.{e}.down_proj.weight", (H, I))
        si = I * c["n_shared_experts"]
        w(p + "mlp.shared_experts.gate_proj.weight", (si, H))
        w(p + "mlp.shared_experts.up_proj.weight", (si, H))
        w(p + "mlp.shared_experts.down_proj.weight", (H, si))
    model_dir.mkdir(parents=True, exist_ok=True)
    (model_dir / "config.json").write_text(json.dumps(c))
    write_safetensors(model_dir / "model.safetensors",
                      {k: (("bfloat16", bf16_bits(v)) if k in bf else ("float32", v))
                       for k, v in vals.items()})
    return vals


def layer_specs(vals: dict[str, np.ndarray]) -> list[LayerSpec]:
    """fp32 layer specs grouped like the reference loader's GLM-4 MoE layers."""
    c = CONFIG
    specs = []
    for layer in range(c["num_hidden_layers"]):
        p = f"model.layers.{layer}."
        is_moe = layer >= c["first_k_dense_replace"]
        names = (sorted(k[len(p):] for k in vals if k.startswith(p)) if is_moe
                 else [n for n in _DENSE_ORDER if p + n in vals])
        meta, off = [], 0
        for n in names:
            nb = vals[p + n].size * 4
            meta.append({"name": n, "shape": list(vals[p + n].shape), "dtype": "float32",
                         "offset": off, "nbytes": nb})
            off += nb
        specs.append(LayerSpec(layer, f"model.layers.{layer}", off,
                               {"tensors": meta, "full_prefix": p, "is_moe": is_moe}))
    return specs


def layer_tensors(vals: dict[str, np.ndarray], layer: int) -> dict[str, np.ndarray]:
    p = f"model.layers.{layer}."
    return {k[len(p):]: v for k, v in vals.items() if k.startswith(p)}
