"""GLM-4 MoE (Glm4MoeForCausalLM) executor with the MoE block on sm_100a.

Constructor and attribute names follow offload_runtime/executors/glm4_moe.py:70-84;
the MoE block (glm4_moe.py:176-240) runs through libmoe_sm100, and so do the
dense MLP of ``first_k_dense_replace`` layers (``metadata["is_moe"] == False``,
glm4_moe.py:102-106, 166-172) and the attention block (glm4_moe.py:112-162),
unless ``dense_mlp`` / ``attention`` delegates are given.
"""
from __future__ import annotations

from typing import Any

from ..config import MoeLayerConfig
from ._device_moe import DeviceMoeExecutor


class GLM4MoeExecutor(DeviceMoeExecutor):
    """Routing modes: ``score_func="softmax"`` (default) reproduces the reference
    executor (softmax of logits + e_score_correction_bias, glm4_moe.py:181-200);
    ``score_func="sigmoid"`` is the HF GLM-4.x rule (sigmoid scores, bias for
    selection only)."""

    family = "glm"

    def __init__(self, config: dict[str, Any], **kw: Any) -> None:
        self.hidden_size: int = config["hidden_size"]
        self.intermediate_size: int = config.get("intermediate_size", 0)
        self.moe_intermediate_size: int = config.get("moe_intermediate_size", self.intermediate_size)
        self.rms_norm_eps: float = config.get("rms_norm_eps", 1e-5)
        self.num_experts_per_tok: int = config.get("num_experts_per_tok", 8)
        self.n_routed_experts: int = config.get("n_routed_experts", 160)
        self.routed_scaling_factor: float = config.get("routed_scaling_factor", 2.5)
        self.norm_topk_prob: bool = config.get("norm_topk_prob", True)
        super().__init__(config, **kw)

    def _parse(self, config: dict[str, Any], overrides: dict[str, Any]) -> MoeLayerConfig:
        return MoeLayerConfig.glm4_moe(config, **overrides)

    def _is_moe_layer(self, layer: Any) -> bool:
        return bool(layer.metadata.get("is_moe", False))

    def _device_attention_config(self) -> Any:
        """Without an ``attention=`` delegate the attention block
        (glm4_moe.py:112-162) runs on the device too (moe_sm100.attention)."""
        if "num_attention_heads" not in self.config:
            return None
        from ..attention import AttentionConfig
        return AttentionConfig.glm4_moe(self.config, max_tokens=self.max_tokens, device=self.device)
