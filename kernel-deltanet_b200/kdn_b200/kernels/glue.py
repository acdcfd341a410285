"""Element-wise steps of the hybrid block on libkdn (one pass each; CUDA tensors only).

``rms_norm`` (layers/hybrid_kernel_deltanet_block.py:23-25), ``swiglu_product`` (silu(gate) * up,
:45-46) and ``mixer_inputs`` (split of the fused q|k|v|beta projection: unit-norm q, k per head,
v, beta = sigmoid, decay = sigmoid(logit_decay) per head) -- the C entries kdn_rmsnorm,
kdn_swiglu and kdn_mixer_inputs -- and ``decode_attention`` (the anchors' one-token attention over
their KV cache, kdn_decode_attention).  Errors raise RuntimeError; there is no CPU path.
"""

from __future__ import annotations

from typing import Optional

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


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float):
    """(h, RMSNorm(h)) with h = x + residual, in one pass (kdn_add_rmsnorm); h is rounded to x's dtype
    as a separate add would leave it."""
    _cuda(x, residual, weight)
    if residual.shape != x.shape or residual.dtype != x.dtype:
        raise RuntimeError("residual must match x in shape and dtype")
    xc, rc = x.contiguous(), residual.contiguous()
    h, out = torch.empty_like(xc), torch.empty_like(xc)
    d = xc.shape[-1]
    w = weight.contiguous()
    _lib.check(_lib.load().kdn_add_rmsnorm(xc.data_ptr(), rc.data_ptr(), _lib.dtype_code(xc), w.data_ptr(),
                                           _lib.dtype_code(w), h.data_ptr(), out.data_ptr(), xc.numel() // d, d, eps,
                                           _lib.stream_handle(x.device)),
               "kdn_add_rmsnorm")
    return h, out


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


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lengths: torch.Tensor,
                     workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q [B, H, 64], caches [>=B, H, max_len, 64], lengths [B] int64 (device) -> softmax(q K^T / 8) V over
    positions [0, lengths[b]] of cache row b, [B, H, 64] in q's dtype (kdn_decode_attention)."""
    _cuda(q, k_cache, v_cache, lengths)
    B, H, dh = q.shape
    max_len = k_cache.shape[2]
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()) or k_cache.dtype != q.dtype:
        raise RuntimeError("k_cache / v_cache must be contiguous and of q's dtype")
    lib = _lib.load()
    need = int(lib.kdn_decode_attention_workspace_size(B, H, max_len))
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need // 4, 1), device=q.device, dtype=torch.float32)
    qc = q.contiguous()
    lc = lengths.to(torch.int64).contiguous()
    out = torch.empty_like(qc)
    _lib.check(lib.kdn_decode_attention(qc.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), lc.data_ptr(),
                                        out.data_ptr(), _lib.dtype_code(qc), B, H, max_len, dh, workspace.data_ptr(),
                                        need, _lib.stream_handle(q.device)), "kdn_decode_attention")
    return out
