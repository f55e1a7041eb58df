"""Layer-blob packer that keeps 16-bit / INT8 expert weights.

The reference loader packs every tensor of a layer into one contiguous blob,
sorted by name, each converted to ``compute_dtype`` (fp32 for bf16 checkpoints:
loader/huggingface.py:492-506, loader/safetensors_storage.py:116-122), and
describes it with ``metadata["tensors"] = [{name, shape, dtype, offset, nbytes}]``.
This packer writes the same description but can keep expert weights as
``bfloat16`` or as per-output-row ``int8`` plus an fp16 ``<name>_scale`` tensor,
so the resident device copy is 2x / 4x smaller than the fp32 blob.
Offsets are aligned (256 B by default) so every tensor is naturally aligned.
"""
from __future__ import annotations

import re
from typing import Any

import numpy as np

# expert, shared-expert and dense-MLP (first_k_dense_replace layers) projections
EXPERT_WEIGHT = re.compile(
    r"(^|\.)mlp\.((experts\.\d+|shared_experts?)\.)?(gate|up|down)_proj\.weight$")


def is_expert_weight(name: str) -> bool:
    return EXPERT_WEIGHT.search(name) is not None


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rounded = ((u.astype(np.uint64) + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        rounded = np.where(nan, np.uint16(0x7FC0), rounded)
    return rounded.reshape(np.shape(a))


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def quantize_int8_per_channel(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric per-output-row INT8 (one fp16 scale per row of an ``[out, in]`` matrix).

    ``scale = fp16(max|row| / 127)``; ``q = clip(rint(w / f32(scale)), -127, 127)``;
    a row whose scale rounds to 0 stores zeros.  Extends the scalar
    ``(q - zero_point) * scale`` format of offload_runtime/quantize.py:24-50.
    """
    w = np.asarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("per-channel quantisation expects a 2-D [out, in] matrix")
    scale = (np.abs(w).max(axis=1) / np.float32(127.0)).astype(np.float16)
    if not np.all(np.isfinite(scale)):
        raise ValueError("row scale overflows float16")
    s32 = scale.astype(np.float32)
    div = np.where(s32 > 0, s32, np.float32(1.0))[:, None]
    q = np.clip(np.rint(w / div), -127, 127)
    q[s32 == 0] = 0
    return q.astype(np.int8), scale


def dequantize_int8_per_channel(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    return q.astype(np.float32) * scale.astype(np.float32)[:, None]


def pack_layer(tensors: dict[str, np.ndarray], expert_format: str = "float32", align: int = 256,
               quantized: dict[str, tuple[np.ndarray, np.ndarray]] | None = None
               ) -> tuple[bytearray, list[dict[str, Any]]]:
    """Pack named arrays into ``(blob, metadata["tensors"])``.

    ``expert_format``: "float32" (reference layout), "bfloat16" or "int8".  For
    "int8", ``quantized`` may supply precomputed ``(q, scale)`` per weight name.
    Non-expert tensors (router, bias, norms, attention) stay fp32.
    """
    if expert_format not in ("float32", "bfloat16", "int8"):
        raise ValueError(f"unknown expert_format {expert_format!r}")
    parts: list[tuple[str, np.ndarray, str]] = []
    for name in sorted(tensors):
        arr = np.asarray(tensors[name])
        if is_expert_weight(name) and expert_format == "bfloat16":
            parts.append((name, bf16_bits(arr), "bfloat16"))
        elif is_expert_weight(name) and expert_format == "int8":
            if quantized is not None and name in quantized:
                q, s = quantized[name]
            else:
                q, s = quantize_int8_per_channel(arr)
            parts.append((name, np.ascontiguousarray(q, dtype=np.int8), "int8"))
            parts.append((name + "_scale", np.ascontiguousarray(s, dtype=np.float16), "float16"))
        else:
            parts.append((name, np.ascontiguousarray(arr, dtype=np.float32), "float32"))
    meta: list[dict[str, Any]] = []
    offset = 0
    for name, arr, dt in parts:
        offset = (offset + align - 1) // align * align
        meta.append({"name": name, "shape": list(arr.shape), "dtype": dt, "offset": offset,
                     "nbytes": int(arr.nbytes)})
        offset += arr.nbytes
    blob = bytearray(offset)
    for (name, arr, _dt), m in zip(parts, meta):
        blob[m["offset"]:m["offset"] + m["nbytes"]] = arr.tobytes()
    return blob, meta
