"""Device buffer reuse plus expert-weight residency.

``DeviceBufferPool`` keeps the reference's size-keyed free list
(offload_runtime/buffer_pool.py:9-30).  ``ResidentLayerPool`` adds residency:
a layer marked resident keeps its device blob across forwards instead of being
freed after ``run_layer`` (runtime.py:180), so its packed MoE weights stay in
HBM and later passes skip storage, H2D and packing for it.  A byte budget bounds
what stays resident (e.g. ~170 GB of a 180 GB B200); least-recently-used
layers are evicted first.
"""
from __future__ import annotations

from collections import OrderedDict, defaultdict
from typing import Any, Callable

from .types import DeviceBuffer


class DeviceBufferPool:
    def __init__(self, backend: Any) -> None:
        self._backend = backend
        self._free: dict[int, list[DeviceBuffer]] = defaultdict(list)

    def acquire(self, nbytes: int) -> DeviceBuffer:
        pool = self._free.get(nbytes)
        if pool:
            return pool.pop()
        return self._backend.alloc_device(nbytes)

    def release(self, buf: DeviceBuffer) -> None:
        self._free[buf.nbytes].append(buf)

    def drain(self) -> None:
        for pool in self._free.values():
            for buf in pool:
                self._backend.free_device(buf)
            pool.clear()
        self._free.clear()


class ResidentLayerPool:
    """Layer-id keyed device blobs that outlive one forward pass."""

    def __init__(self, backend: Any, budget_bytes: int,
                 on_evict: Callable[[int], None] | None = None) -> None:
        self._backend = backend
        self.budget_bytes = budget_bytes
        self._on_evict = on_evict
        self._layers: OrderedDict[int, DeviceBuffer] = OrderedDict()
        self.resident_bytes = 0

    def is_resident(self, layer_id: int) -> bool:
        return layer_id in self._layers

    def get(self, layer_id: int) -> DeviceBuffer | None:
        buf = self._layers.get(layer_id)
        if buf is not None:
            self._layers.move_to_end(layer_id)
        return buf

    def admit(self, layer_id: int, buf: DeviceBuffer) -> bool:
        """Keep ``buf`` resident; returns False (caller frees it) if it cannot fit."""
        if buf.nbytes > self.budget_bytes:
            return False
        while self.resident_bytes + buf.nbytes > self.budget_bytes and self._layers:
            self.evict(next(iter(self._layers)))
        self._layers[layer_id] = buf
        self.resident_bytes += buf.nbytes
        return True

    def evict(self, layer_id: int) -> None:
        buf = self._layers.pop(layer_id, None)
        if buf is None:
            return
        self.resident_bytes -= buf.nbytes
        if self._on_evict is not None:
            self._on_evict(layer_id)
        self._backend.free_device(buf)

    def drain(self) -> None:
        for lid in list(self._layers):
            self.evict(lid)
