"""Kernel-DeltaNet layer surface -- drop-in for layers/kernel_deltanet_layer.py.

``KernelDeltaNetLayer.forward(q, k, v, beta, state=None, decay=None)`` takes
per-head queries/keys/values [B, H, T, d_k|d_v] and gates [B, H, T] and returns
``(y [B, H, T, d_v], S [B, H, d_v, D])``: the exact delta rule with the
structured-FWHT lift (the computation of kernels/fused_kernel_deltanet.py:31-155,
reached from the layer level the way pipeline/transmute.py:65-89 does it:
heads flattened into the batch, one chunked scan).  ``state`` is the carried
recurrent state; passing the returned state back continues the sequence
exactly (a prefill split in two equals one pass).  ``KernelTTTLayer`` is the
reference's alias (layers/kernel_deltanet_layer.py:147).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from ..kernels.fused_kernel_deltanet import fused_chunked_deltanet_forward
from ..kernels.fwht import FastWalshHadamardProjection


class KernelDeltaNetLayer(nn.Module):
    def __init__(self, num_heads: int, d_k: int = 64, d_v: int = 64, rkhs_dim: int = 512, chunk_size: int = 64,
                 seed: int = 42, mode: Optional[str] = None):
        super().__init__()
        self.num_heads = num_heads
        self.d_k = d_k
        self.d_v = d_v
        self.rkhs_dim = rkhs_dim
        self.chunk_size = chunk_size
        self.mode = mode
        self.fwht_proj = FastWalshHadamardProjection(d_k=d_k, D=rkhs_dim, seed=seed)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                state: Optional[torch.Tensor] = None,
                decay: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        B, H, T, d_k = q.shape
        if H != self.num_heads:
            raise RuntimeError(f"got {H} heads, layer has {self.num_heads}")
        dv = v.shape[-1]
        D = self.rkhs_dim
        flat = lambda t, w: t.reshape(B * H, T, w)  # noqa: E731
        S0 = None if state is None else state.reshape(B * H, dv, D)
        y, S = fused_chunked_deltanet_forward(
            flat(q, d_k), flat(k, d_k), flat(v, dv), beta.reshape(B * H, T),
            None if decay is None else decay.reshape(B * H, T), self.fwht_proj, self.chunk_size, S0,
            mode=self.mode)
        return y.view(B, H, T, dv), S.view(B, H, dv, D)


KernelTTTLayer = KernelDeltaNetLayer
