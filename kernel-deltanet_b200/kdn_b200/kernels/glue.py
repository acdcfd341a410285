"""Element-wise steps of the hybrid block on libkdn (one pass each; CUDA tensors only).

``linear`` (the block's bias-free projections, kdn_linear), ``rms_norm``
(layers/hybrid_kernel_deltanet_block.py:23-25), ``swiglu_product`` (silu(gate) * up,
:45-46) and ``mixer_inputs`` (split of the fused q|k|v|beta projection: unit-norm q, k per head,
v, beta = sigmoid, decay = sigmoid(logit_decay) per head) -- the C entries kdn_rmsnorm,
kdn_swiglu and kdn_mixer_inputs -- and the anchors' attention: ``anchor_qkv`` (rotary q/k and the KV-cache
fill, kdn_anchor_qkv), ``varlen_causal_attention`` (packed causal prefill, kdn_varlen_causal_attention) and
``decode_attention`` (one token over the cache, kdn_decode_attention).  Errors raise RuntimeError; there is no CPU path.
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


def mixer_inputs(z: torch.Tensor, num_heads: int, logit_decay: torch.Tensor, d_head: int = 64,
                 cu_seqlens: Optional[torch.Tensor] = None):
    """z [n, 3 H d_head + H] (rows may be strided, as a padded projection output leaves them) ->
    q, k (unit norm), v [n, H, d_head] in z's dtype; beta, decay [n, H] fp32.  With cu_seqlens (device
    int64 [B + 1]) the same-shaped outputs hold the head-major per-sequence layout (sequence i's head h
    at rows cu[i] H + h T_i ...), the layout the ragged prefill consumes."""
    _cuda(z, logit_decay)
    zc = z if (z.dim() == 2 and z.stride(1) == 1) else z.contiguous()
    n, H = zc.shape[0], num_heads
    if zc.shape[1] != 3 * H * d_head + H:
        raise RuntimeError(f"z has {zc.shape[1]} columns, expected {3 * H * d_head + H}")
    q = torch.empty(n, H, d_head, device=z.device, dtype=z.dtype)
    k, v = torch.empty_like(q), torch.empty_like(q)
    beta = torch.empty(n, H, device=z.device, dtype=torch.float32)
    decay = torch.empty_like(beta)
    ld = logit_decay.contiguous()
    cu = cu_seqlens.to(torch.int64).contiguous() if cu_seqlens is not None else None
    _lib.check(_lib.load().kdn_mixer_inputs(zc.data_ptr(), _lib.dtype_code(zc), n, H, d_head,
                                            zc.stride(0) if n > 1 else 0, ld.data_ptr(), _lib.dtype_code(ld),
                                            cu.data_ptr() if cu is not None else None,
                                            cu.numel() - 1 if cu is not None else 0, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                            beta.data_ptr(), decay.data_ptr(), _lib.stream_handle(z.device)),
               "kdn_mixer_inputs")
    return q, k, v, beta, decay


def linear(x: torch.Tensor, weight: torch.Tensor, out_dtype: Optional[torch.dtype] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [..., K] @ weight[N, K]^T on libkdn (kdn_linear: GEMV up to 64 rows, tcgen05 GEMM above), bf16
    operands, fp32 accumulation, output in out_dtype (x's dtype by default; bf16 or fp32).  When N is not
    a multiple of 16 bytes of output the rows are padded and the result is a strided view.  `out`: a
    contiguous [M, N] tensor (rows 16-byte aligned) to write into instead."""
    _cuda(x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise RuntimeError("kdn linear takes bf16 operands")
    out_dtype = out_dtype or x.dtype
    K = x.shape[-1]
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise RuntimeError(f"weight is {tuple(weight.shape)}, x has {K} columns")
    xc = x.reshape(-1, K)
    if not xc.is_contiguous() or xc.data_ptr() % 16:
        xc = xc.contiguous()
    wc = weight if weight.is_contiguous() else weight.contiguous()
    M = xc.shape[0]
    if out is not None:
        if out.shape != (M, N) or not out.is_contiguous() or out.dtype != out_dtype:
            raise RuntimeError(f"out must be a contiguous [{M}, {N}] {out_dtype} tensor")
        buf, ldo = out, N
    else:
        per16 = 16 // torch.empty((), dtype=out_dtype).element_size()
        ldo = (N + per16 - 1) // per16 * per16
        buf = torch.empty(M, ldo, device=x.device, dtype=out_dtype)
    _lib.check(_lib.load().kdn_linear(xc.data_ptr(), wc.data_ptr(), buf.data_ptr(), _lib.dtype_code(buf), M, N, K,
                                      ldo, _lib.stream_handle(x.device)), "kdn_linear")
    out = buf if ldo == N else buf[:, :N]
    return out if x.dim() == 2 else out.reshape(*x.shape[:-1], N)


def swiglu_interleave(w_gate_up: torch.Tensor) -> torch.Tensor:
    """[2 d_ff, K] (gate rows, then up rows) -> the row-block interleaved layout kdn_linear_swiglu reads
    (128 gate rows, the same 128 up rows, ...)."""
    f2, K = w_gate_up.shape
    f = f2 // 2
    if f2 % 256:
        raise RuntimeError("d_ff must be a multiple of 128")
    return w_gate_up.view(2, f // 128, 128, K).transpose(0, 1).reshape(f2, K).contiguous()


def linear_swiglu(x: torch.Tensor, w_interleaved: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """silu(x W_gate^T) * (x W_up^T), [M, d_ff] bf16, from the interleaved weight (kdn_linear_swiglu: the
    product is formed in the GEMM epilogue)."""
    _cuda(x, w_interleaved)
    if x.dtype != torch.bfloat16 or w_interleaved.dtype != torch.bfloat16:
        raise RuntimeError("kdn linear_swiglu takes bf16 operands")
    xc = x if (x.is_contiguous() and x.data_ptr() % 16 == 0) else x.contiguous()
    M, K = xc.shape
    f = w_interleaved.shape[0] // 2
    if out is None:
        out = torch.empty(M, f, device=x.device, dtype=torch.bfloat16)
    elif out.shape != (M, f) or not out.is_contiguous() or out.dtype != torch.bfloat16:
        raise RuntimeError(f"out must be a contiguous [{M}, {f}] bf16 tensor")
    _lib.check(_lib.load().kdn_linear_swiglu(xc.data_ptr(), w_interleaved.data_ptr(), out.data_ptr(), M, f, K, f,
                                             _lib.stream_handle(x.device)), "kdn_linear_swiglu")
    return out


def anchor_qkv(qkv: torch.Tensor, cu_seqlens: torch.Tensor, num_heads: int, rope_theta: float,
               k_cache: torch.Tensor, v_cache: torch.Tensor, cache_rows: Optional[torch.Tensor] = None,
               start_pos: Optional[torch.Tensor] = None, q_head_major: bool = True) -> torch.Tensor:
    """qkv [n, 3 H 64] (bf16, q | k | v) of sequences packed by cu_seqlens (device int64 [B + 1]) -> rotated
    q ([H, n, 64] head-major, or [n, H, 64]); rotated k and v are stored into the caches [rows, H, L, 64] at
    position (t - cu[i] + start_pos[i]) of row cache_rows[i] (kdn_anchor_qkv)."""
    _cuda(qkv, cu_seqlens, k_cache, v_cache)
    n, H = qkv.shape[0], num_heads
    if qkv.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise RuntimeError("anchor_qkv takes bf16 tensors")
    if qkv.numel() != n * 3 * H * 64 or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise RuntimeError("qkv must be [n, 3 H 64]; caches contiguous [rows, H, L, 64]")
    qc = qkv.contiguous()
    cu = cu_seqlens.to(torch.int64).contiguous()
    rows = cache_rows.to(torch.int64).contiguous() if cache_rows is not None else None
    start = start_pos.to(torch.int64).contiguous() if start_pos is not None else None
    q = torch.empty((H, n, 64) if q_head_major else (n, H, 64), device=qkv.device, dtype=qkv.dtype)
    _lib.check(_lib.load().kdn_anchor_qkv(qc.data_ptr(), _lib.dtype_code(qc), cu.data_ptr(),
                                          start.data_ptr() if start is not None else None,
                                          rows.data_ptr() if rows is not None else None, cu.numel() - 1, n, H, 64,
                                          float(rope_theta), q.data_ptr(), int(q_head_major), k_cache.data_ptr(),
                                          v_cache.data_ptr(), k_cache.shape[0], k_cache.shape[2],
                                          _lib.stream_handle(qkv.device)), "kdn_anchor_qkv")
    return q


def varlen_causal_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cu_seqlens: torch.Tensor,
                            max_seqlen: int, cache_rows: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Head-major q [H, n, 64] of packed sequences (cu_seqlens device int64 [B + 1], every length <= max_seqlen)
    against their cache rows -> causal softmax(q K^T / 8) V, [n, H, 64] bf16 (kdn_varlen_causal_attention)."""
    _cuda(q, k_cache, v_cache, cu_seqlens)
    H, n, dh = q.shape
    if not (q.is_contiguous() and k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise RuntimeError("q and the caches must be contiguous")
    cu = cu_seqlens.to(torch.int64).contiguous()
    rows = cache_rows.to(torch.int64).contiguous() if cache_rows is not None else None
    out = torch.empty(n, H, dh, device=q.device, dtype=q.dtype)
    _lib.check(_lib.load().kdn_varlen_causal_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                                       _lib.dtype_code(q), cu.data_ptr(),
                                                       rows.data_ptr() if rows is not None else None, cu.numel() - 1,
                                                       n, H, dh, k_cache.shape[0], k_cache.shape[2], int(max_seqlen),
                                                       out.data_ptr(), _lib.stream_handle(q.device)),
               "kdn_varlen_causal_attention")
    return out


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
