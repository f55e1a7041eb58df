"""Qwen3-Next (Qwen3NextForCausalLM) executor with the MoE block on sm_100a.

Constructor and attribute names follow offload_runtime/executors/qwen3_next.py:105-133.
Every layer runs the MoE block (qwen3_next.py:156): softmax top-k without bias
or scale, plus the shared expert gated by ``sigmoid(h . w_gate)``
(qwen3_next.py:321-331).  Attention (Gated DeltaNet / gated GQA) is delegated.
"""
from __future__ import annotations

from typing import Any

from ..config import MoeLayerConfig
from ._device_moe import DeviceMoeExecutor


class Qwen3NextExecutor(DeviceMoeExecutor):
    family = "qwen3"

    def __init__(self, config: dict[str, Any], **kw: Any) -> None:
        self.hidden_size: int = config["hidden_size"]
        self.rms_norm_eps: float = config.get("rms_norm_eps", 1e-6)
        self.num_experts: int = config.get("num_experts", config.get("n_routed_experts", 512))
        self.num_experts_per_tok: int = config.get("num_experts_per_tok", 10)
        self.moe_intermediate_size: int = config.get("moe_intermediate_size", 512)
        self.shared_expert_intermediate_size: int = config.get(
            "shared_expert_intermediate_size", self.moe_intermediate_size)
        self.norm_topk_prob: bool = config.get("norm_topk_prob", True)
        super().__init__(config, **kw)

    def _parse(self, config: dict[str, Any], overrides: dict[str, Any]) -> MoeLayerConfig:
        return MoeLayerConfig.qwen3_next(config, **overrides)
