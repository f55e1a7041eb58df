"""Layer / buffer descriptors with the reference's field names.

Same fields and meaning as offload_runtime/types.py:7-41 (``LayerSpec``,
``HostBuffer``, ``DeviceBuffer``), so objects made by the reference loader and
runtime can be handed to this package unchanged (attribute access only).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any


@dataclass(frozen=True, slots=True)
class LayerSpec:
    layer_id: int
    name: str
    nbytes: int
    metadata: dict[str, Any] = field(default_factory=dict)


@dataclass(slots=True)
class HostBuffer:
    view: memoryview
    pinned: bool = False

    @property
    def nbytes(self) -> int:
        return self.view.nbytes


@dataclass(slots=True)
class DeviceBuffer:
    handle: Any      # CUDA device pointer (int) for the "cuda" backend
    nbytes: int
    backend: str
