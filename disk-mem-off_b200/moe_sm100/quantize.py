"""Per-channel INT8 for the runtime's dequantizer hook.

The runtime calls a dequantizer before the H2D copy of a layer
(offload_runtime/runtime.py:147-151) through the protocol of
offload_runtime/quantize.py:14-21 (``needs_dequantize`` / ``dequantize`` /
``decompressed_nbytes``).  The reference's own scalar dequantizers
(``Int8Dequantizer``, ``Float16Dequantizer``, ``CompositeDequantizer``,
offload_runtime/quantize.py:24-97) stay where they are; this module adds one
more implementation of that protocol, which a ``CompositeDequantizer`` can list.

``Int8PerChannelDequantizer`` handles layers packed by ``moe_sm100.packing`` with
``expert_format="int8"`` (``metadata["dtype"] == "int8_per_channel"``).  With
``keep_on_device=True`` (default) it reports ``needs_dequantize() == False`` so the
runtime copies the compressed blob as-is and the sm_100a kernels dequantize
inside the GEMM tile load.  ``dequantize()`` still produces the fp32 blob the
reference executor expects, for runtimes that want host-side expansion.
"""
from __future__ import annotations

from typing import Any, Protocol

import numpy as np

from .packing import dequantize_int8_per_channel
from .types import HostBuffer, LayerSpec


class Dequantizer(Protocol):
    def needs_dequantize(self, layer: LayerSpec) -> bool: ...

    def dequantize(self, layer: LayerSpec, buf: HostBuffer) -> HostBuffer: ...

    def decompressed_nbytes(self, layer: LayerSpec) -> int: ...


class Int8PerChannelDequantizer:
    """Per-output-row INT8 expert weights with fp16 ``<name>_scale`` tensors."""

    def __init__(self, keep_on_device: bool = True) -> None:
        self.keep_on_device = keep_on_device

    @staticmethod
    def is_per_channel(layer: LayerSpec) -> bool:
        return layer.metadata.get("dtype") == "int8_per_channel"

    def needs_dequantize(self, layer: LayerSpec) -> bool:
        return self.is_per_channel(layer) and not self.keep_on_device

    def decompressed_nbytes(self, layer: LayerSpec) -> int:
        if not self.needs_dequantize(layer):
            return layer.nbytes
        total = 0
        for m in layer.metadata["tensors"]:
            if m["name"].endswith("_scale"):
                continue
            total += int(np.prod(m["shape"])) * 4
        return total

    def dequantize(self, layer: LayerSpec, buf: HostBuffer) -> HostBuffer:
        if not self.needs_dequantize(layer):
            return buf
        raw = buf.view.cast("B")
        metas = {m["name"]: m for m in layer.metadata["tensors"]}
        out_meta: list[dict[str, Any]] = []
        parts: list[bytes] = []
        offset = 0
        for m in layer.metadata["tensors"]:
            name = m["name"]
            if name.endswith("_scale"):
                continue
            a = np.frombuffer(raw, dtype=np.dtype(m["dtype"]) if m["dtype"] != "bfloat16" else np.uint16,
                              count=int(np.prod(m["shape"])), offset=int(m["offset"])).reshape(m["shape"])
            if m["dtype"] == "int8":
                s = metas[name + "_scale"]
                sc = np.frombuffer(raw, dtype=np.float16, count=int(np.prod(s["shape"])),
                                   offset=int(s["offset"]))
                f = dequantize_int8_per_channel(a, sc)
            elif m["dtype"] == "bfloat16":
                f = (a.astype(np.uint32) << 16).view(np.float32)
            else:
                f = a.astype(np.float32)
            b = f.tobytes()
            out_meta.append({"name": name, "shape": list(f.shape), "dtype": "float32",
                             "offset": offset, "nbytes": len(b)})
            parts.append(b)
            offset += len(b)
        layer.metadata["dequantized_tensors"] = out_meta
        return HostBuffer(view=memoryview(bytearray(b"".join(parts))), pinned=False)
