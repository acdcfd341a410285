"""Element-wise steps of the hybrid block on libkdn (one pass each; CUDA tensors only).

``rms_norm`` (layers/hybrid_kernel_deltanet_block.py:23-25), ``swiglu_product`` (silu(gate) * up,
:45-46) and ``mixer_inputs`` (split of the fused q|k|v|beta projection: unit-norm q, k per head,
v, beta = sigmoid, decay = sigmoid(logit_decay) per head) -- the C entries kdn_rmsnorm,
kdn_swiglu and kdn_mixer_inputs.  Errors raise RuntimeError; there is no CPU path.
"""

from __future__ import annotations

import torch

from .. import _lib


def _cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("kdn_b200 runs on CUDA tensors only (no CPU fallback)")


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    _cuda(x, weight)
    xc = x.contiguous()
    out = torch.empty_like(xc)
    d = xc.shape[-1]
    w = weight.contiguous()
    _lib.check(_lib.load().kdn_rmsnorm(xc.data_ptr(), _lib.dtype_code(xc), w.data_ptr(), _lib.dtype_code(w),
                                       out.data_ptr(), xc.numel() // d, d, eps, _lib.stream_handle(x.device)),
               "kdn_rmsnorm")
    return out


def swiglu_product(gate_up: torch.Tensor) -> torch.Tensor:
    """[n, 2 d_ff] (gate columns first) -> silu(gate) * up [n, d_ff]."""
    _cuda(gate_up)
    g = gate_up.contiguous()
    f = g.shape[-1] // 2
    out = torch.empty(*g.shape[:-1], f, device=g.device, dtype=g.dtype)
    _lib.check(_lib.load().kdn_swiglu(g.data_ptr(), out.data_ptr(), _lib.dtype_code(g), g.numel() // (2 * f), f,
                                      _lib.stream_handle(g.device)), "kdn_swiglu")
    return out


def mixer_inputs(z: torch.Tensor, num_heads: int, logit_decay: torch.Tensor, d_head: int = 64):
    """z [n, 3 H d_head + H] -> q, k (unit norm), v [n, H, d_head] in z's dtype; beta, decay [n, H] fp32."""
    _cuda(z, logit_decay)
    zc = z.contiguous()
    n, H = zc.shape[0], num_heads
    if zc.shape[1] != 3 * H * d_head + H:
        raise RuntimeError(f"z has {zc.shape[1]} columns, expected {3 * H * d_head + H}")
    q = torch.empty(n, H, d_head, device=z.device, dtype=z.dtype)
    k, v = torch.empty_like(q), torch.empty_like(q)
    beta = torch.empty(n, H, device=z.device, dtype=torch.float32)
    decay = torch.empty_like(beta)
    ld = logit_decay.contiguous()
    _lib.check(_lib.load().kdn_mixer_inputs(zc.data_ptr(), _lib.dtype_code(zc), n, H, d_head, ld.data_ptr(),
                                            _lib.dtype_code(ld), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                            beta.data_ptr(), decay.data_ptr(), _lib.stream_handle(z.device)),
               "kdn_mixer_inputs")
    return q, k, v, beta, decay
