"""kdn_b200 -- B200 (sm_100a) implementation of the Kernel-DeltaNet hot path.

Host-side mirror of the reference surfaces for this path:

    kdn_b200.kernels.fwht.FastWalshHadamardProjection         (kernels/fwht.py)
    kdn_b200.kernels.fused_kernel_deltanet.*                  (kernels/fused_kernel_deltanet.py)
    kdn_b200.layers.kernel_deltanet_layer.KernelDeltaNetLayer (layers/kernel_deltanet_layer.py)
    kdn_b200.serving.vllm_kernel_deltanet_op.*                (serving/vllm_kernel_deltanet_op.cpp)
    kdn_b200.serving.ragged.ragged_prefill                    (serving/vllm_ragged_batching.py)
    kdn_b200.kernels.blelloch_scan.*                          (kernels/blelloch_scan.py)
    kdn_b200.distributed                                      (one process per GPU: independent
                                                               scans, or one sequence in blocks)

All compute goes through libkdn.so (C ABI in include/kdn.h).
"""

from ._lib import LIB_PATH, load
from .distributed import sequence_parallel_prefill, shard_range
from .kernels import (FastWalshHadamardProjection, FusedKernelDeltaNet, blelloch_prefix_scan, chunk_block_transition,
                      chunked_deltanet_backward, compose_transitions, fused_chunked_deltanet_forward,
                      sequential_prefix_scan)
from .layers import KernelDeltaNetLayer, KernelTTTLayer
from .serving import fork_recurrent_state, hybrid_recurrent_forward, ragged_prefill
from .models import HybridCache, KernelDeltaNetLM

__all__ = ["load", "LIB_PATH", "FastWalshHadamardProjection", "fused_chunked_deltanet_forward",
           "chunked_deltanet_backward",
           "FusedKernelDeltaNet", "KernelDeltaNetLayer", "KernelTTTLayer", "hybrid_recurrent_forward",
           "fork_recurrent_state", "compose_transitions", "blelloch_prefix_scan", "sequential_prefix_scan",
           "chunk_block_transition", "sequence_parallel_prefill", "shard_range", "ragged_prefill",
           "KernelDeltaNetLM", "HybridCache"]
