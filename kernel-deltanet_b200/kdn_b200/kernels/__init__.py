"""Hot-path kernels (mirror of the reference's kernels/ package surface for this path)."""

from .blelloch_scan import (blelloch_prefix_scan, chunk_block_transition, compose_transitions, prefix_states,
                            sequential_prefix_scan)
from .fwht import FastWalshHadamardProjection
from .fused_kernel_deltanet import (FusedKernelDeltaNet, FusedKernelDeltaNetFunction, chunked_deltanet_backward,
                                    fused_chunked_deltanet_forward)

__all__ = ["FastWalshHadamardProjection", "fused_chunked_deltanet_forward", "chunked_deltanet_backward", "FusedKernelDeltaNet",
           "FusedKernelDeltaNetFunction", "compose_transitions", "blelloch_prefix_scan", "sequential_prefix_scan",
           "prefix_states", "chunk_block_transition"]
