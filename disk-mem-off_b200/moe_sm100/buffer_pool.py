"""Expert-weight residency for the offload runtime.

The reference runtime frees every layer's device weights after ``run_layer``
(offload_runtime/runtime.py:180) and copies them again on the next forward.
``ResidentLayerPool`` is the accounting side of keeping them: a layer admitted
here stays on the device (its packed MoE weights in HBM) across forwards, so later
passes skip storage, the H2D copy and packing for it.  A byte budget bounds what
stays resident (for example ~170 GB of a 180 GB B200); the least recently used
layer is released first.  What "releasing" means belongs to the owner of the
device memory (the executor's packed plan, a device blob), so each layer is
admitted with the callable that frees it.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Callable


class ResidentLayerPool:
    """Layer-id keyed device residency with a byte budget and LRU release."""

    def __init__(self, budget_bytes: int, on_evict: Callable[[int], None] | None = None) -> None:
        self.budget_bytes = int(budget_bytes)
        self._on_evict = on_evict
        self._layers: OrderedDict[int, tuple[int, Callable[[], None]]] = OrderedDict()
        self.resident_bytes = 0

    def __contains__(self, layer_id: int) -> bool:
        return layer_id in self._layers

    def is_resident(self, layer_id: int) -> bool:
        return layer_id in self._layers

    def touch(self, layer_id: int) -> bool:
        """Mark a resident layer as just used; False if it is not resident."""
        if layer_id not in self._layers:
            return False
        self._layers.move_to_end(layer_id)
        return True

    def admit(self, layer_id: int, nbytes: int, release: Callable[[], None]) -> bool:
        """Keep a layer of ``nbytes`` resident, releasing older layers to make room.

        Returns False, without releasing anything, when the layer alone exceeds
        the budget; the caller then frees it itself."""
        nbytes = int(nbytes)
        if layer_id in self._layers:
            self.evict(layer_id)
        if nbytes > self.budget_bytes:
            return False
        while self._layers and self.resident_bytes + nbytes > self.budget_bytes:
            self.evict(next(iter(self._layers)))
        self._layers[layer_id] = (nbytes, release)
        self.resident_bytes += nbytes
        return True

    def evict(self, layer_id: int) -> None:
        entry = self._layers.pop(layer_id, None)
        if entry is None:
            return
        nbytes, release = entry
        self.resident_bytes -= nbytes
        release()
        if self._on_evict is not None:
            self._on_evict(layer_id)

    def drain(self) -> None:
        for lid in list(self._layers):
            self.evict(lid)
