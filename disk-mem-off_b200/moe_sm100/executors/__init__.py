from ._device_moe import DeviceMoeExecutor, reference_delegates
from .glm4_moe import GLM4MoeExecutor
from .qwen3_next import Qwen3NextExecutor

__all__ = ["DeviceMoeExecutor", "GLM4MoeExecutor", "Qwen3NextExecutor", "reference_delegates"]
