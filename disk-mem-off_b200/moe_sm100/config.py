"""MoE-block configuration, parsed from the HF ``config.json`` dict the way the
reference executors do (glm4_moe.py:70-84, qwen3_next.py:105-133)."""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any

from . import _lib

SCORE_FUNCS = {"softmax": _lib.MOE_SCORE_SOFTMAX, "sigmoid": _lib.MOE_SCORE_SIGMOID}
WEIGHT_FORMATS = {"f16": _lib.MOE_WEIGHTS_F16, "bf16": _lib.MOE_WEIGHTS_F16,
                  "int8": _lib.MOE_WEIGHTS_INT8_PC, "int8_pc": _lib.MOE_WEIGHTS_INT8_PC}


@dataclass(frozen=True)
class MoeLayerConfig:
    hidden: int
    n_experts: int
    top_k: int
    inter: int
    shared_inter: int = 0
    score_func: str = "softmax"      # "softmax" = reference rule, "sigmoid" = HF GLM-4.x rule
    norm_topk_prob: bool = True
    use_bias: bool = True            # add e_score_correction_bias when the layer has one
    has_shared_gate: bool = False    # Qwen3 sigmoid(h . w_gate) on the shared expert
    weight_format: str = "f16"       # "f16" (bf16-valued weights) or "int8" per-channel
    routed_scaling_factor: float = 1.0
    rms_norm_eps: float = 1e-6
    max_tokens: int = 4096
    device: int = 0
    expert_begin: int = 0            # expert parallel: this rank's share [begin, end)
    expert_end: int = 0              # 0, 0 = all experts

    def to_c(self) -> _lib.MoeConfigC:
        if self.score_func not in SCORE_FUNCS:
            raise ValueError(f"score_func must be one of {sorted(SCORE_FUNCS)}")
        if self.weight_format not in WEIGHT_FORMATS:
            raise ValueError(f"weight_format must be one of {sorted(WEIGHT_FORMATS)}")
        return _lib.MoeConfigC(
            hidden=self.hidden, n_experts=self.n_experts, top_k=self.top_k, inter=self.inter,
            shared_inter=self.shared_inter, score_func=SCORE_FUNCS[self.score_func],
            norm_topk_prob=int(self.norm_topk_prob), use_bias=int(self.use_bias),
            has_shared_gate=int(self.has_shared_gate),
            weight_format=WEIGHT_FORMATS[self.weight_format],
            routed_scaling_factor=float(self.routed_scaling_factor),
            rms_norm_eps=float(self.rms_norm_eps), max_tokens=self.max_tokens,
            expert_begin=self.expert_begin, expert_end=self.expert_end, device=self.device)

    def with_shapes(self, inter: int, shared_inter: int, has_shared_gate: bool) -> "MoeLayerConfig":
        return replace(self, inter=inter, shared_inter=shared_inter, has_shared_gate=has_shared_gate)

    # -- constructors mirroring the reference executors' config parsing --
    @classmethod
    def glm4_moe(cls, config: dict[str, Any], **overrides: Any) -> "MoeLayerConfig":
        """glm4_moe.py:70-84 defaults."""
        inter = config.get("moe_intermediate_size", config.get("intermediate_size", 0))
        n_shared = config.get("n_shared_experts", 1)
        kw = dict(hidden=config["hidden_size"],
                  n_experts=config.get("n_routed_experts", 160),
                  top_k=config.get("num_experts_per_tok", 8),
                  inter=inter, shared_inter=inter * n_shared if n_shared else 0,
                  norm_topk_prob=config.get("norm_topk_prob", True),
                  routed_scaling_factor=config.get("routed_scaling_factor", 2.5),
                  rms_norm_eps=config.get("rms_norm_eps", 1e-5), use_bias=True,
                  has_shared_gate=False)
        kw.update(overrides)
        return cls(**kw)

    @classmethod
    def dense_mlp(cls, config: dict[str, Any], **overrides: Any) -> "MoeLayerConfig":
        """The dense MLP of GLM-4 first_k_dense_replace layers (glm4_moe.py:166-172):
        a plan with no routed experts whose mlp.{gate,up,down}_proj run as the
        shared-expert GEMMs (``intermediate_size`` columns)."""
        kw = dict(hidden=config["hidden_size"], n_experts=0, top_k=0, inter=0,
                  shared_inter=config["intermediate_size"], use_bias=False,
                  has_shared_gate=False, routed_scaling_factor=1.0,
                  rms_norm_eps=config.get("rms_norm_eps", 1e-5))
        kw.update(overrides)
        return cls(**kw)

    @classmethod
    def qwen3_next(cls, config: dict[str, Any], **overrides: Any) -> "MoeLayerConfig":
        """qwen3_next.py:105-133 defaults (softmax top-k, no bias, no scale)."""
        inter = config.get("moe_intermediate_size", 512)
        kw = dict(hidden=config["hidden_size"],
                  n_experts=config.get("num_experts", config.get("n_routed_experts", 512)),
                  top_k=config.get("num_experts_per_tok", 10), inter=inter,
                  shared_inter=config.get("shared_expert_intermediate_size", inter),
                  norm_topk_prob=config.get("norm_topk_prob", True),
                  routed_scaling_factor=1.0, rms_norm_eps=config.get("rms_norm_eps", 1e-6),
                  use_bias=False, has_shared_gate=True, score_func="softmax")
        kw.update(overrides)
        return cls(**kw)
