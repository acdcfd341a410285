"""Hot-path kernels (mirror of the reference's kernels/ package surface for this path)."""

from .fwht import FastWalshHadamardProjection
from .fused_kernel_deltanet import FusedKernelDeltaNet, FusedKernelDeltaNetFunction, fused_chunked_deltanet_forward

__all__ = ["FastWalshHadamardProjection", "fused_chunked_deltanet_forward", "FusedKernelDeltaNet",
           "FusedKernelDeltaNetFunction"]
