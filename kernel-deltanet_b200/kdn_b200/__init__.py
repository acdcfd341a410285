"""kdn_b200 -- B200 (sm_100a) implementation of the Kernel-DeltaNet hot path.

Host-side mirror of the reference surfaces for this path:

    kdn_b200.kernels.fwht.FastWalshHadamardProjection         (kernels/fwht.py)
    kdn_b200.kernels.fused_kernel_deltanet.*                  (kernels/fused_kernel_deltanet.py)
    kdn_b200.layers.kernel_deltanet_layer.KernelDeltaNetLayer (layers/kernel_deltanet_layer.py)
    kdn_b200.serving.vllm_kernel_deltanet_op.*                (serving/vllm_kernel_deltanet_op.cpp)

All compute goes through libkdn.so (C ABI in include/kdn.h).
"""

from ._lib import LIB_PATH, load
from .kernels import FastWalshHadamardProjection, FusedKernelDeltaNet, fused_chunked_deltanet_forward
from .layers import KernelDeltaNetLayer, KernelTTTLayer
from .serving import fork_recurrent_state, hybrid_recurrent_forward

__all__ = ["load", "LIB_PATH", "FastWalshHadamardProjection", "fused_chunked_deltanet_forward",
           "FusedKernelDeltaNet", "KernelDeltaNetLayer", "KernelTTTLayer", "hybrid_recurrent_forward",
           "fork_recurrent_state"]
