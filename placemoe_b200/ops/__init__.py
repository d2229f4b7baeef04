"""sm_100a ops with PyTorch reference paths for CPU tensors."""

from ._ext import available, check_device_error, device_error, kernels, p2p_status
from .gemm import gemm_nn, gemm_nt, gemm_tn, linear

__all__ = ["available", "check_device_error", "device_error", "kernels", "p2p_status", "gemm_nn", "gemm_nt", "gemm_tn", "linear"]
