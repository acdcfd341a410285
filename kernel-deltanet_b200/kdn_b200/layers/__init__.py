from .hybrid_kernel_deltanet_block import (HybridKernelDeltaNetBlock, HybridKernelTTTBlock, KernelDeltaNetMixer,
                                           RMSNorm, SoftmaxAnchor, SwiGLUFFN)
from .kernel_deltanet_layer import KernelDeltaNetLayer, KernelTTTLayer

__all__ = ["KernelDeltaNetLayer", "KernelTTTLayer", "HybridKernelDeltaNetBlock", "HybridKernelTTTBlock",
           "KernelDeltaNetMixer", "RMSNorm", "SoftmaxAnchor", "SwiGLUFFN"]
