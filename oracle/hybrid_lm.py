"""Oracle: hybrid Kernel-DeltaNet LM forward in float64 (TEST INFRASTRUCTURE ONLY).

Restates, for one sequence at a time, the model that kdn_b200.models.kernel_deltanet_lm runs:

    x = Embed(ids)                                            models/kernel_deltanet_lm.py:107
    per block:  h = x + Mixer(RMSNorm(x)); x = h + SwiGLU(RMSNorm(h))
                                                              layers/hybrid_kernel_deltanet_block.py:85-96
    logits = LMHead(RMSNorm(x))                               models/kernel_deltanet_lm.py:113-114

RMSNorm is x * rsqrt(mean(x^2) + eps) * w (hybrid_kernel_deltanet_block.py:23-25) and SwiGLU
W_down(silu(x W_gate) * (x W_up)) (:45-46).  The Kernel-DeltaNet mixer projects q, k, v and beta,
normalises q and k per head (layers/kernel_deltanet_layer.py:98-99), takes beta = sigmoid(.)
(serving/tensor_parallel_runner.py:62) and the per-head retention sigmoid(logit_decay)
(kernel_deltanet_layer.py:71-73) as every token's decay, and runs the chunked delta rule of
``oracle.chunked.chunked_deltanet_forward`` (pinned to the reference's golden vectors).  Anchor
layers are causal softmax attention with rotate-half rotary positions
(models/upcycling_llama_bridge.py:138-140), scale 1/sqrt(d_head).

``params`` is a plain dict of float64 arrays:
    {"embed": [V, d], "final_norm": [d], "lm_head": [V, d],
     "layers": [{"anchor": bool, "norm1": [d], "norm2": [d], "w_gate_up": [2 f, d], "w_down": [d, f],
                 "w_qkvb": [3 H dh + H, d], "logit_decay": [H], "w_out": [d, H dh]      (Kernel-DeltaNet)
                 | "w_qkv": [3 H dh, d], "w_out": [d, H dh]}, ...]}                      (anchor)
"""

from __future__ import annotations

import numpy as np

from .chunked import chunked_deltanet_forward
from .projection import ProjectionConstants


def rms_norm(x, w, eps=1e-6):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def swiglu(x, w_gate_up, w_down):
    f = w_down.shape[1]
    z = x @ w_gate_up.T
    g, u = z[..., :f], z[..., f:]
    return (g / (1.0 + np.exp(-g)) * u) @ w_down.T


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _normalize(x):  # torch.nn.functional.normalize (eps 1e-12)
    return x / np.maximum(np.linalg.norm(x, axis=-1, keepdims=True), 1e-12)


def kdn_mixer(x, p, H: int, dh: int, consts: ProjectionConstants, chunk: int):
    T = x.shape[0]
    z = x @ p["w_qkvb"].T
    q = _normalize(z[:, :H * dh].reshape(T, H, dh))
    k = _normalize(z[:, H * dh:2 * H * dh].reshape(T, H, dh))
    v = z[:, 2 * H * dh:3 * H * dh].reshape(T, H, dh)
    beta = _sigmoid(z[:, 3 * H * dh:])  # [T, H]
    decay = np.broadcast_to(_sigmoid(p["logit_decay"])[:, None], (H, T))
    y, _ = chunked_deltanet_forward(q.transpose(1, 0, 2), k.transpose(1, 0, 2), v.transpose(1, 0, 2), beta.T,
                                    np.ascontiguousarray(decay), consts, chunk)
    return y.transpose(1, 0, 2).reshape(T, H * dh) @ p["w_out"].T


def rotary(x, pos, theta):
    d = x.shape[-1]
    inv = theta ** (-np.arange(0, d, 2, dtype=np.float64) / d)
    ang = pos[:, None].astype(np.float64) * inv[None, :]
    cos = np.concatenate([np.cos(ang), np.cos(ang)], axis=-1)[:, None, :]
    sin = np.concatenate([np.sin(ang), np.sin(ang)], axis=-1)[:, None, :]
    rot = np.concatenate([-x[..., d // 2:], x[..., :d // 2]], axis=-1)
    return x * cos + rot * sin


def anchor_attention(x, p, H: int, dh: int, theta: float):
    T = x.shape[0]
    q, k, v = (x @ p["w_qkv"].T).reshape(T, 3, H, dh).transpose(1, 0, 2, 3)
    pos = np.arange(T)
    q, k = rotary(q, pos, theta), rotary(k, pos, theta)
    s = np.einsum("thd,uhd->htu", q, k) / np.sqrt(dh)
    s = np.where(np.tril(np.ones((T, T), bool))[None], s, -np.inf)
    s = np.exp(s - s.max(axis=-1, keepdims=True))
    a = s / s.sum(axis=-1, keepdims=True)
    o = np.einsum("htu,uhd->thd", a, v)
    return o.reshape(T, H * dh) @ p["w_out"].T


def lm_logits(params: dict, ids, num_heads: int, consts: ProjectionConstants, chunk: int = 64,
              rope_theta: float = 10000.0, eps: float = 1e-6) -> np.ndarray:
    """Logits [T, V] of every position of one sequence `ids` [T]."""
    x = params["embed"][np.asarray(ids)]
    d = x.shape[-1]
    dh = d // num_heads
    for p in params["layers"]:
        h = rms_norm(x, p["norm1"], eps)
        mixed = (anchor_attention(h, p, num_heads, dh, rope_theta) if p["anchor"]
                 else kdn_mixer(h, p, num_heads, dh, consts, chunk))
        h = x + mixed
        x = h + swiglu(rms_norm(h, p["norm2"], eps), p["w_gate_up"], p["w_down"])
    return rms_norm(x, params["final_norm"], eps) @ params["lm_head"].T


def greedy(params: dict, prompt, steps: int, num_heads: int, consts: ProjectionConstants, chunk: int = 64,
           rope_theta: float = 10000.0, eps: float = 1e-6) -> list:
    """Greedy continuation of `prompt` by `steps` tokens, re-running the whole sequence each step
    (models/kernel_deltanet_lm.py:187-196 with temperature 0)."""
    seq = list(int(t) for t in prompt)
    out = []
    for _ in range(steps):
        nxt = int(np.argmax(lm_logits(params, seq, num_heads, consts, chunk, rope_theta, eps)[-1]))
        out.append(nxt)
        seq.append(nxt)
    return out
