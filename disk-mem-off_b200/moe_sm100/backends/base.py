"""Vendor-neutral device contract, same methods as offload_runtime/backends/base.py:9-77."""
from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any

from ..types import DeviceBuffer, HostBuffer


class DeviceBackend(ABC):
    name: str

    @abstractmethod
    def create_stream(self, purpose: str) -> Any: ...

    @abstractmethod
    def destroy_stream(self, stream: Any) -> None: ...

    @abstractmethod
    def alloc_device(self, nbytes: int) -> DeviceBuffer: ...

    @abstractmethod
    def free_device(self, buf: DeviceBuffer) -> None: ...

    @property
    def supports_pinned_host(self) -> bool:
        return False

    @property
    def supports_peer_to_peer(self) -> bool:
        return False

    @property
    def supports_graph_capture(self) -> bool:
        return False

    def alloc_pinned_host(self, nbytes: int) -> HostBuffer:
        raise NotImplementedError(f"{self.name} does not support pinned host memory")

    def free_pinned_host(self, buf: HostBuffer) -> None:
        raise NotImplementedError(f"{self.name} does not support pinned host memory")

    @abstractmethod
    def copy_h2d_async(self, dst: DeviceBuffer, src: HostBuffer, stream: Any) -> None: ...

    @abstractmethod
    def copy_d2h_async(self, dst: HostBuffer, src: DeviceBuffer, stream: Any) -> None: ...

    @abstractmethod
    def record_event(self, stream: Any) -> Any: ...

    @abstractmethod
    def destroy_event(self, event: Any) -> None: ...

    @abstractmethod
    def wait_event(self, stream: Any, event: Any) -> None: ...

    @abstractmethod
    def synchronize_stream(self, stream: Any) -> None: ...
