from .cuda_backend import CUDABackend

__all__ = ["CUDABackend"]
