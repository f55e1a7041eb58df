from .base import DeviceBackend
from .cuda_backend import CUDABackend

__all__ = ["CUDABackend", "DeviceBackend"]
