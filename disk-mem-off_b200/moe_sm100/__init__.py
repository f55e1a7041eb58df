"""moe_sm100: B200 (sm_100a) MoE feed-forward block for disk-mem-off executors.

Public surface:
  MoeLayerConfig, MoeLayer                 -- one resident layer over the C ABI
  executors.GLM4MoeExecutor / Qwen3NextExecutor  -- drop-in executor MoE path
  backends.CUDABackend                     -- ctypes DeviceBackend over libmoe_sm100
  packing.pack_layer                       -- bf16 / int8-preserving layer blobs
  quantize.*                               -- Dequantizer protocol + per-channel INT8
  buffer_pool.ResidentLayerPool            -- expert-weight residency
"""
from .config import MoeLayerConfig
from .layer import MoeLayer

__all__ = ["MoeLayer", "MoeLayerConfig"]
__version__ = "0.1.0"
