"""Pre-norm hybrid decoder block: Kernel-DeltaNet mixer (or a softmax-attention anchor) + SwiGLU.

Mirrors layers/hybrid_kernel_deltanet_block.py of the reference:
    h   = x + Mixer(RMSNorm(x))                       (:85-89)
    out = h + SwiGLU(RMSNorm(h))                      (:91-96)
with RMSNorm(x) = x * rsqrt(mean(x^2) + eps) * w    (:23-25, eps 1e-6)
and  SwiGLU(x)  = W_down(silu(x W_gate) * (x W_up)) (:45-46).

The blocks run on packed token batches (serving layout): a prefill takes the tokens of
several sequences back to back, [total_tokens, d_model], with ``cu_seqlens``; a decode
step takes one token per sequence, [num_seqs, d_model].  Per-sequence recurrent state
lives in a slot pool owned by the caller (the model's cache).

Mixers:
* ``KernelDeltaNetMixer`` -- the hot path.  One GEMM gives q, k, v (H heads of 64) and the
  write strength beta (the column-parallel projections of serving/tensor_parallel_runner.py:41-44,
  fused); q, k are L2-normalised per head (layers/kernel_deltanet_layer.py:98-99), beta =
  sigmoid(.) (tensor_parallel_runner.py:62), and the per-head retention lambda =
  sigmoid(logit_decay) (kernel_deltanet_layer.py:60-62, :71-73) is the decay of every token.
  Prefill runs ``ragged_prefill`` (libkdn chunked prefill, states written into the pool) and
  decode runs ``hybrid_recurrent_forward`` (libkdn decode step, read-out before the update),
  both through the FWHT feature lift d_k = 64 -> D = 512.
* ``SoftmaxAnchor`` -- the full-attention anchor layers the reference keeps at fixed depths of
  its hybrid models (models/upcycling_llama_bridge.py:240-249, anchors at [10, 21]):
  multi-head causal softmax attention with rotary positions (the retained Llama attention,
  rotate-half convention, models/upcycling_llama_bridge.py:138-140) and a KV cache for decode.
  With bf16 weights the rotary q/k and the KV-cache fill are one libkdn kernel (kdn_anchor_qkv), the
  packed causal prefill is libkdn's tcgen05 varlen attention (kdn_varlen_causal_attention) and the
  one-token decode its split-K kdn_decode_attention, which reads only each sequence's live keys; the
  fp32 verification mode runs torch's rotary and SDPA.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from ..kernels import glue
from ..kernels.fwht import FastWalshHadamardProjection
from ..serving.ragged import ragged_prefill
from ..serving.vllm_kernel_deltanet_op import hybrid_recurrent_forward


class Linear(nn.Linear):
    """Bias-free projection (the nn.Linear(bias=False) layers of layers/kernel_deltanet_layer.py:46-49 and
    layers/hybrid_kernel_deltanet_block.py:43-45).  bf16 weights run on libkdn's kdn_linear (a GEMV
    kernel for decode-size batches, the TMA-fed tcgen05 GEMM for prefill), with no other path; fp32
    weights -- the exact-arithmetic verification mode -- use torch's fp32 matmul."""

    def __init__(self, in_features: int, out_features: int):
        super().__init__(in_features, out_features, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.weight.dtype == torch.bfloat16:
            return glue.linear(x, self.weight)
        return F.linear(x, self.weight)


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight, formed in fp32 in one pass (kdn_rmsnorm)
    (layers/hybrid_kernel_deltanet_block.py:16-25)."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return glue.rms_norm(x, self.weight, self.eps)

    def add_forward(self, x: torch.Tensor, residual: torch.Tensor):
        """(h, RMSNorm(h)) with h = x + residual: the residual add and the norm after it in one pass."""
        return glue.add_rms_norm(x, residual, self.weight, self.eps)


class SwiGLUFFN(nn.Module):
    """W_down(silu(x W_gate) * (x W_up)) (layers/hybrid_kernel_deltanet_block.py:28-46); the gate and
    up projections are one GEMM ([2 d_ff, d_model] weight, gate rows first).  Long token batches are
    processed in row blocks of `chunk_tokens` to bound the [tokens, 2 d_ff] intermediate."""

    def __init__(self, d_model: int, d_ff: Optional[int] = None, chunk_tokens: int = 65536):
        super().__init__()
        if d_ff is None:  # 8/3 expansion rounded up to 64 (the reference default, :38-42)
            d_ff = (int(d_model * 8 / 3) + 63) // 64 * 64
        self.d_ff = d_ff
        self.chunk_tokens = chunk_tokens
        self.w_gate_up = Linear(d_model, 2 * d_ff)
        self.w_down = Linear(d_ff, d_model)

    def _interleaved(self) -> torch.Tensor:
        """The gate/up weight in the row-block interleaved layout of kdn_linear_swiglu (rebuilt when the
        parameter changes)."""
        w = self.w_gate_up.weight
        key = (w.data_ptr(), w._version, w.dtype)
        if getattr(self, "_il_key", None) != key:
            self._il = glue.swiglu_interleave(w.detach())
            self._il_key = key
        return self._il

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        n = x.shape[0]
        if self.w_gate_up.weight.dtype == torch.bfloat16 and x.dim() == 2 and n > 64 and self.d_ff % 128 == 0:
            # prefill: silu(gate) * up formed in the gate/up GEMM's epilogue, the down projection written
            # straight into its rows of the output
            w_il = self._interleaved()
            out = torch.empty(n, self.w_down.out_features, device=x.device, dtype=x.dtype)
            for s in range(0, n, self.chunk_tokens):
                glue.linear(glue.linear_swiglu(x[s:s + self.chunk_tokens], w_il), self.w_down.weight,
                            out=out[s:s + self.chunk_tokens])
            return out
        if n <= self.chunk_tokens:
            return self.w_down(glue.swiglu_product(self.w_gate_up(x)))
        out = torch.empty_like(x)
        for s in range(0, n, self.chunk_tokens):
            out[s:s + self.chunk_tokens] = self.w_down(glue.swiglu_product(self.w_gate_up(x[s:s + self.chunk_tokens])))
        return out


class KernelDeltaNetMixer(nn.Module):
    """Multi-head Kernel-DeltaNet sequence mixer on the libkdn prefill / decode kernels."""

    def __init__(self, d_model: int, num_heads: int, d_head: int = 64, rkhs_dim: int = 512, chunk_size: int = 64,
                 initial_decay: float = 0.99, seed: int = 42, mode: Optional[str] = None):
        super().__init__()
        self.num_heads, self.d_head, self.chunk_size, self.mode = num_heads, d_head, chunk_size, mode
        hd = num_heads * d_head
        self.w_qkvb = Linear(d_model, 3 * hd + num_heads)  # q | k | v | beta rows
        init_logit = math.log(initial_decay / (1.0 - initial_decay + 1e-7))
        self.logit_decay = nn.Parameter(torch.full((num_heads,), float(init_logit)))
        self.w_out = Linear(hd, d_model)
        self.fwht = FastWalshHadamardProjection(d_head, rkhs_dim, seed)

    def project(self, x: torch.Tensor):
        """x [n, d_model] -> q, k [n, H, d_head] (unit norm), v [n, H, d_head], beta, decay [n, H] (fp32)."""
        return glue.mixer_inputs(self.w_qkvb(x), self.num_heads, self.logit_decay, self.d_head)

    def prefill(self, x: torch.Tensor, cu_seqlens: torch.Tensor, states: torch.Tensor, slots: torch.Tensor,
                fresh: torch.Tensor) -> torch.Tensor:
        """Packed prefill: every sequence starts from a zero state where `fresh` (else from its slot)
        and leaves its final state in `states[slots[i]]`."""
        # q, k, v, beta, decay come out in the head-major per-sequence layout the prefill reads
        q, k, v, beta, decay = glue.mixer_inputs(self.w_qkvb(x), self.num_heads, self.logit_decay, self.d_head,
                                                 cu_seqlens=cu_seqlens)
        y = torch.empty_like(v)
        ragged_prefill(q, k, v, beta, decay, cu_seqlens, states, slots, y, self.fwht, self.chunk_size,
                       mode=self.mode, initial_state_mask=~fresh, head_major_inputs=True)
        return self.w_out(y.view(x.shape[0], -1))

    def decode(self, x: torch.Tensor, states: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
        """One token per sequence: read out with the state before the token, then update it in place."""
        q, k, v, beta, decay = self.project(x)
        y = torch.empty_like(v)
        hybrid_recurrent_forward(q, k, v, beta, decay, states, slots, y, self.fwht)
        return self.w_out(y.view(x.shape[0], -1))


# SDPA back ends for the anchors: flash (then memory-efficient) for the causal prefill, memory-efficient
# for the masked one-token decode when the libkdn decode attention (d_head 64) does not apply.  cuDNN's back end is left out: it builds a new graph (with a device
# query of tens of milliseconds) for every new sequence length, which made the host the bottleneck.
_PREFILL_BACKENDS = [SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]
_DECODE_BACKENDS = [SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]


def rotary(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotate-half rotary embedding of x [n, H, d] at integer positions pos [n] (computed in fp32)."""
    d = x.shape[-1]
    inv = theta ** (-torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d)
    ang = pos.to(torch.float32)[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1)[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1)[:, None, :]
    xf = x.float()
    rot = torch.cat([-xf[..., d // 2:], xf[..., :d // 2]], dim=-1)
    return (xf * cos + rot * sin).to(x.dtype)


class SoftmaxAnchor(nn.Module):
    """Causal multi-head softmax attention with rotary positions and a per-sequence KV cache."""

    def __init__(self, d_model: int, num_heads: int, d_head: int = 64, rope_theta: float = 10000.0):
        super().__init__()
        self.num_heads, self.d_head, self.rope_theta = num_heads, d_head, rope_theta
        self.w_qkv = Linear(d_model, 3 * num_heads * d_head)
        self.w_out = Linear(num_heads * d_head, d_model)

    def _qkv(self, x: torch.Tensor, pos: torch.Tensor):
        n, H, dh = x.shape[0], self.num_heads, self.d_head
        q, k, v = self.w_qkv(x).view(n, 3, H, dh).unbind(1)
        return rotary(q, pos, self.rope_theta), rotary(k, pos, self.rope_theta), v

    def _native(self, x: torch.Tensor, k_cache: torch.Tensor) -> bool:
        """bf16 activations and caches with 64-wide heads run on libkdn's anchor kernels."""
        return x.dtype == torch.bfloat16 and k_cache.dtype == torch.bfloat16 and self.d_head == 64

    def prefill(self, x: torch.Tensor, cu: list, k_cache: torch.Tensor, v_cache: torch.Tensor,
                rows: list, cu_dev: Optional[torch.Tensor] = None) -> torch.Tensor:
        """cu: host list of sequence offsets (cu_dev: the same on the device, if the caller has it);
        sequence i is written to cache row rows[i] from position 0."""
        n = x.shape[0]
        if self._native(x, k_cache):
            if n == 0:
                return self.w_out(x.new_empty(0, self.num_heads * self.d_head))
            B = len(cu) - 1
            cu_t = cu_dev if cu_dev is not None else torch.tensor(cu, device=x.device, dtype=torch.int64)
            rows_t = None if list(rows) == list(range(B)) else torch.tensor(rows, device=x.device, dtype=torch.int64)
            q = glue.anchor_qkv(self.w_qkv(x), cu_t, self.num_heads, self.rope_theta, k_cache, v_cache, rows_t)
            max_len = max(cu[i + 1] - cu[i] for i in range(B))
            o = glue.varlen_causal_attention(q, k_cache, v_cache, cu_t, max_len, rows_t)
            return self.w_out(o.view(n, -1))
        # fp32 verification mode: torch rotary and SDPA per sequence
        pos = torch.cat([torch.arange(cu[i + 1] - cu[i], device=x.device) for i in range(len(cu) - 1)]) \
            if n else torch.zeros(0, dtype=torch.int64, device=x.device)
        q, k, v = self._qkv(x, pos)
        o = torch.empty_like(q)
        for i in range(len(cu) - 1):
            s, e = cu[i], cu[i + 1]
            if e == s:
                continue
            qi, ki, vi = (t[s:e].transpose(0, 1).unsqueeze(0) for t in (q, k, v))  # [1, H, T, d]
            with sdpa_kernel(_PREFILL_BACKENDS):
                o[s:e] = F.scaled_dot_product_attention(qi, ki, vi, is_causal=True)[0].transpose(0, 1)
            k_cache[rows[i], :, :e - s] = ki[0]
            v_cache[rows[i], :, :e - s] = vi[0]
        return self.w_out(o.view(n, -1))

    def decode(self, x: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lengths: torch.Tensor,
               span: int) -> torch.Tensor:
        """Token b of the step sits at position lengths[b] (device tensor) of cache row b and attends to
        positions [0, lengths[b]]; `span` is a host bound on max(lengths) + 1 (the key range read).  No
        host synchronisation: the step can be captured in a CUDA graph."""
        B = x.shape[0]
        if self._native(x, k_cache) and k_cache.shape[0] == B:
            cu = torch.arange(B + 1, device=x.device, dtype=torch.int64)  # one token per sequence
            q = glue.anchor_qkv(self.w_qkv(x), cu, self.num_heads, self.rope_theta, k_cache, v_cache,
                                start_pos=lengths, q_head_major=False)
            return self.w_out(glue.decode_attention(q, k_cache, v_cache, lengths).reshape(B, -1))
        q, k, v = self._qkv(x, lengths)
        rows = torch.arange(B, device=x.device)
        k_cache[rows, :, lengths] = k
        v_cache[rows, :, lengths] = v
        if self.d_head == 64 and k_cache.shape[0] == B and q.dtype in (torch.float32, torch.bfloat16):
            o = glue.decode_attention(q, k_cache, v_cache, lengths)  # split-K over the live lengths only
        else:
            mask = (torch.arange(span, device=x.device)[None, :] <= lengths[:, None])[:, None, None, :]
            with sdpa_kernel(_DECODE_BACKENDS):
                o = F.scaled_dot_product_attention(q.unsqueeze(2), k_cache[:B, :, :span], v_cache[:B, :, :span],
                                                   attn_mask=mask)
        return self.w_out(o.reshape(B, -1))


class HybridKernelDeltaNetBlock(nn.Module):
    """Pre-norm residual block; `anchor=True` swaps the Kernel-DeltaNet mixer for softmax attention."""

    def __init__(self, d_model: int, num_heads: int, d_ff: Optional[int] = None, anchor: bool = False,
                 chunk_size: int = 64, mode: Optional[str] = None, rope_theta: float = 10000.0,
                 norm_eps: float = 1e-6):
        super().__init__()
        self.anchor = anchor
        self.norm1 = RMSNorm(d_model, norm_eps)
        d_head = d_model // num_heads
        self.mixer = (SoftmaxAnchor(d_model, num_heads, d_head, rope_theta) if anchor
                      else KernelDeltaNetMixer(d_model, num_heads, d_head, chunk_size=chunk_size, mode=mode))
        self.norm2 = RMSNorm(d_model, norm_eps)
        self.ffn = SwiGLUFFN(d_model, d_ff)

    def finish(self, x: torch.Tensor, mixed: torch.Tensor) -> torch.Tensor:
        h = x + mixed
        return h + self.ffn(self.norm2(h))


# reference aliases (layers/hybrid_kernel_deltanet_block.py:101-106)
HybridKernelTTTBlock = HybridKernelDeltaNetBlock
