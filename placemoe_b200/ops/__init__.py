"""sm_100a ops with PyTorch reference paths for CPU tensors."""

from ._ext import available, check_device_error, device_error, kernels
from .gemm import gemm_nn, gemm_nt, gemm_tn, linear

__all__ = ["available", "check_device_error", "device_error", "kernels", "gemm_nn", "gemm_nt", "gemm_tn", "linear"]
