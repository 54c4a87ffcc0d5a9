"""Native B200 kernels behind the flash-eq API (libflasheq_b200.so via a C ABI)."""
from .block_diagonal import CUDANotAvailableError, block_diagonal_cuda

__all__ = ["block_diagonal_cuda", "CUDANotAvailableError"]
