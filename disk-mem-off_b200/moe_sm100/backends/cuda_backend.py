"""CUDA backend as a thin ctypes layer over libmoe_sm100's runtime entry points.

It satisfies the reference's ``DeviceBackend`` contract
(offload_runtime/backends/base.py:9-77) by its methods alone, so the reference
runtime accepts it without this package importing the reference.  Same class
name, methods and error behaviour as offload_runtime/backends/cuda_backend.py:35-128 (status != 0 -> ``RuntimeError``,
host buffer too small -> ``ValueError``, read-only host view -> ``ValueError``),
but bound to ``moe_rt_*`` in libmoe_sm100.so instead of cuda-python, so the
device pointers it hands out are the ones the MoE entry points consume.
"""
from __future__ import annotations

import ctypes
from ctypes import byref, c_int32, c_void_p
from typing import Any

from .._lib import check, lib
from ..types import DeviceBuffer, HostBuffer


def _ptr_from_writable_view(view: memoryview) -> int:
    if view.readonly:
        raise ValueError(
            "HostBuffer.view must be writable for async cudaMemcpyAsync. "
            "Use pinned writable host buffers in production.")
    return ctypes.addressof(ctypes.c_char.from_buffer(view))


def _stream(stream: Any) -> c_void_p:
    if stream is None:
        return c_void_p(0)
    if isinstance(stream, c_void_p):
        return stream
    return c_void_p(int(stream))


class CUDABackend:
    name = "cuda"

    def __init__(self, device_id: int = 0) -> None:
        self.device_id = device_id
        check(lib().moe_rt_set_device(device_id))

    @property
    def supports_pinned_host(self) -> bool:
        return True

    @property
    def supports_peer_to_peer(self) -> bool:
        """True when this device can map the memory of at least one other device."""
        for peer in range(self.device_count()):
            if peer == self.device_id:
                continue
            ok = c_int32(0)
            check(lib().moe_rt_can_access_peer(self.device_id, peer, byref(ok)))
            if ok.value:
                return True
        return False

    @property
    def supports_graph_capture(self) -> bool:
        return True

    @staticmethod
    def device_count() -> int:
        n = c_int32(0)
        check(lib().moe_rt_device_count(byref(n)))
        return int(n.value)

    def alloc_pinned_host(self, nbytes: int) -> HostBuffer:
        p = c_void_p()
        check(lib().moe_rt_malloc_host(nbytes, byref(p)))
        arr = (ctypes.c_byte * nbytes).from_address(p.value)
        return HostBuffer(view=memoryview(arr), pinned=True)

    def free_pinned_host(self, buf: HostBuffer) -> None:
        check(lib().moe_rt_free_host(c_void_p(ctypes.addressof(ctypes.c_char.from_buffer(buf.view)))))

    def create_stream(self, purpose: str) -> Any:
        _ = purpose
        s = c_void_p()
        check(lib().moe_rt_stream_create(byref(s)))
        return s

    def destroy_stream(self, stream: Any) -> None:
        check(lib().moe_rt_stream_destroy(_stream(stream)))

    def alloc_device(self, nbytes: int) -> DeviceBuffer:
        p = c_void_p()
        check(lib().moe_rt_malloc(nbytes, byref(p)))
        return DeviceBuffer(handle=int(p.value or 0), nbytes=nbytes, backend=self.name)

    def free_device(self, buf: DeviceBuffer) -> None:
        check(lib().moe_rt_free(c_void_p(int(buf.handle))))

    def copy_h2d_async(self, dst: DeviceBuffer, src: HostBuffer, stream: Any) -> None:
        if src.nbytes < dst.nbytes:
            raise ValueError(f"Host buffer ({src.nbytes}B) smaller than device buffer ({dst.nbytes}B)")
        check(lib().moe_rt_memcpy_h2d_async(c_void_p(int(dst.handle)),
                                            c_void_p(_ptr_from_writable_view(src.view)),
                                            dst.nbytes, _stream(stream)))

    def copy_d2h_async(self, dst: HostBuffer, src: DeviceBuffer, stream: Any) -> None:
        if dst.nbytes < src.nbytes:
            raise ValueError(f"Host buffer ({dst.nbytes}B) smaller than device buffer ({src.nbytes}B)")
        check(lib().moe_rt_memcpy_d2h_async(c_void_p(_ptr_from_writable_view(dst.view)),
                                            c_void_p(int(src.handle)), src.nbytes, _stream(stream)))

    def copy_d2h_range(self, dst: Any, src: DeviceBuffer, offset: int, nbytes: int, stream: Any) -> None:
        """Copy ``nbytes`` at ``offset`` of a device buffer into a writable host array."""
        if offset < 0 or nbytes < 0 or offset + nbytes > src.nbytes:
            raise ValueError("range outside the device buffer")
        mv = memoryview(dst).cast("B")
        if mv.nbytes < nbytes:
            raise ValueError("host array too small")
        check(lib().moe_rt_memcpy_d2h_async(c_void_p(_ptr_from_writable_view(mv)),
                                            c_void_p(int(src.handle) + offset), nbytes,
                                            _stream(stream)))

    def record_event(self, stream: Any) -> Any:
        e = c_void_p()
        check(lib().moe_rt_event_record(_stream(stream), byref(e)))
        return e

    def destroy_event(self, event: Any) -> None:
        check(lib().moe_rt_event_destroy(event))

    def wait_event(self, stream: Any, event: Any) -> None:
        check(lib().moe_rt_stream_wait_event(_stream(stream), event))

    def synchronize_stream(self, stream: Any) -> None:
        check(lib().moe_rt_stream_synchronize(_stream(stream)))
