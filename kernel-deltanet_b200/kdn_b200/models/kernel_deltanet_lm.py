"""Hybrid causal LM on the Kernel-DeltaNet kernels -- mirror of models/kernel_deltanet_lm.py.

The reference LM (models/kernel_deltanet_lm.py:17-197) is an embedding, a stack of pre-norm
blocks, a final RMSNorm and a (tied) LM head; its inference path runs the prompt token by token
(`prefill_and_init_states`, :122-140) and then one recurrent step per generated token
(`generate`, :142-197).  The hybrid models of the reference keep a few softmax-attention
"anchor" layers at fixed depths (models/upcycling_llama_bridge.py:240-249; anchors [10, 21]
of a 22-layer stack, the `hybrid_attn_layers` the evaluations pass).

Here the same model runs as a serving engine over packed, ragged batches:

* ``prefill(input_ids, cu_seqlens, cache)`` -- the prompts of several sequences back to back
  ([total_tokens] int64) -> the next-token logits of every sequence [num_seqs, vocab].  Each
  Kernel-DeltaNet layer is one chunked-prefill pass per sequence (libkdn), which leaves the
  final state in the cache's state pool; each anchor layer fills its KV cache.
* ``decode_step(tokens, cache)`` -- one token per sequence -> logits [num_seqs, vocab]: the
  libkdn decode step (read-out before the update, state updated in place) per Kernel-DeltaNet
  layer, cached attention per anchor layer.
* ``generate`` (same arguments as the reference; temperature 0 is greedy), ``forward``
  (uniform [B, T] batch -> all logits, + cross-entropy with targets) and
  ``prefill_and_init_states`` keep the reference surface.

Weights are initialised as the reference does (:68-79): linear weights N(0, 0.02/sqrt(2 L)),
the embedding N(0, 0.02), RMSNorm weights 1, the LM head tied to the embedding.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..layers.hybrid_kernel_deltanet_block import HybridKernelDeltaNetBlock, Linear, RMSNorm


@dataclass
class HybridCache:
    """Per-sequence inference state of a batch: one fp32 state pool [B, H, d_v, D] per
    Kernel-DeltaNet layer, one K/V cache [B, H, max_len, d_head] per anchor layer, and the number
    of tokens each sequence holds (host list; row b of every pool / cache is sequence b)."""

    states: List[Optional[torch.Tensor]]
    k_cache: List[Optional[torch.Tensor]]
    v_cache: List[Optional[torch.Tensor]]
    lengths: List[int]
    max_len: int
    lengths_dev: Optional[torch.Tensor] = field(default=None)

    @property
    def batch(self) -> int:
        return len(self.lengths)


class KernelDeltaNetLM(nn.Module):
    def __init__(self, vocab_size: int = 32000, d_model: int = 2048, num_layers: int = 22, num_heads: int = 32,
                 d_ff: Optional[int] = 8192, anchor_layers: Sequence[int] = (10, 21), chunk_size: int = 64,
                 rkhs_dim: int = 512, tie_weights: bool = True, mode: Optional[str] = None,
                 rope_theta: float = 10000.0):
        super().__init__()
        if d_model % num_heads:
            raise ValueError(f"d_model ({d_model}) must be divisible by num_heads ({num_heads})")
        self.vocab_size, self.d_model, self.num_layers, self.num_heads = vocab_size, d_model, num_layers, num_heads
        self.d_head = d_model // num_heads
        self.rkhs_dim = rkhs_dim
        self.anchor_layers = sorted(set(int(a) for a in anchor_layers))
        if any(a < 0 or a >= num_layers for a in self.anchor_layers):
            raise ValueError(f"anchor layers {self.anchor_layers} outside [0, {num_layers})")
        self.embed = nn.Embedding(vocab_size, d_model)
        self.layers = nn.ModuleList([
            HybridKernelDeltaNetBlock(d_model, num_heads, d_ff, anchor=(i in self.anchor_layers), chunk_size=chunk_size,
                                      mode=mode, rope_theta=rope_theta)
            for i in range(num_layers)])
        self.final_norm = RMSNorm(d_model)
        self.lm_head = Linear(d_model, vocab_size)
        if tie_weights:
            self.lm_head.weight = self.embed.weight
        self.apply(self._init_weights)

    def _init_weights(self, module):
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=0.02 / math.sqrt(2 * self.num_layers))
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)

    # ------------------------------------------------------------------ cache
    def new_cache(self, batch: int, max_len: int, device=None, dtype: Optional[torch.dtype] = None) -> HybridCache:
        """State pools and KV caches for `batch` sequences of up to `max_len` tokens."""
        p = self.embed.weight
        device = p.device if device is None else device
        dtype = p.dtype if dtype is None else dtype
        states, kc, vc = [], [], []
        for layer in self.layers:
            if layer.anchor:
                states.append(None)
                kc.append(torch.zeros(batch, self.num_heads, max_len, self.d_head, device=device, dtype=dtype))
                vc.append(torch.zeros(batch, self.num_heads, max_len, self.d_head, device=device, dtype=dtype))
            else:
                states.append(torch.zeros(batch, self.num_heads, self.d_head, self.rkhs_dim, device=device,
                                          dtype=torch.float32))
                kc.append(None)
                vc.append(None)
        return HybridCache(states, kc, vc, [0] * batch, max_len)

    # ------------------------------------------------------------------ serving path
    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor, cu_seqlens: Union[torch.Tensor, Sequence[int]],
                cache: HybridCache) -> torch.Tensor:
        """Packed prompts [total_tokens] with offsets cu_seqlens [B + 1] -> next-token logits [B, vocab].
        Sequence i becomes row i of `cache` (its previous contents are replaced)."""
        cu = [int(c) for c in (cu_seqlens.tolist() if torch.is_tensor(cu_seqlens) else cu_seqlens)]
        B = len(cu) - 1
        if B != cache.batch:
            raise ValueError(f"cache holds {cache.batch} sequences, the batch has {B}")
        lens = [cu[i + 1] - cu[i] for i in range(B)]
        if min(lens) < 1 or max(lens) > cache.max_len:
            raise ValueError(f"prompt lengths must be in [1, {cache.max_len}]")
        dev = self.embed.weight.device
        ids = input_ids.to(dev)
        cu_dev = torch.tensor(cu, device=dev, dtype=torch.int64)
        rows = torch.arange(B, device=dev)
        fresh = torch.ones(B, dtype=torch.bool)
        x, delta = self._prefill_body(self.embed(ids), cu, cu_dev, cache, rows, fresh)
        cache.lengths = lens
        cache.lengths_dev = torch.tensor(lens, device=dev, dtype=torch.int64)
        last = cu_dev[1:] - 1
        if delta is None:  # no blocks
            return self.lm_head(self.final_norm(x[last]))
        return self.lm_head(self.final_norm.add_forward(x[last], delta[last])[1])

    def _prefill_body(self, x: torch.Tensor, cu: list, cu_dev: torch.Tensor, cache: HybridCache,
                      rows: torch.Tensor, fresh: torch.Tensor):
        """The blocks over a packed batch; returns (x, delta) with the last FFN output `delta` not yet
        added to the residual stream x (each residual add runs fused with the RMSNorm after it)."""
        B = len(cu) - 1
        delta = None
        for li, layer in enumerate(self.layers):
            if delta is None:
                h = layer.norm1(x)
            else:
                x, h = layer.norm1.add_forward(x, delta)
            if layer.anchor:
                mixed = layer.mixer.prefill(h, cu, cache.k_cache[li], cache.v_cache[li], list(range(B)), cu_dev)
            else:
                mixed = layer.mixer.prefill(h, cu_dev, cache.states[li], rows, fresh)
            x, h = layer.norm2.add_forward(x, mixed)
            delta = layer.ffn(h)
        return x, delta

    def _decode_body(self, tokens: torch.Tensor, cache: HybridCache, span: int) -> torch.Tensor:
        """Device work of one decode step (no host synchronisation; capturable in a CUDA graph)."""
        B = cache.batch
        rows = torch.arange(B, device=tokens.device)
        x = self.embed(tokens)
        delta = None  # the FFN output not yet added to the residual stream x
        for li, layer in enumerate(self.layers):
            # each residual add runs fused with the RMSNorm that follows it
            if delta is None:
                h = layer.norm1(x)
            else:
                x, h = layer.norm1.add_forward(x, delta)
            if layer.anchor:
                mixed = layer.mixer.decode(h, cache.k_cache[li], cache.v_cache[li], cache.lengths_dev, span)
            else:
                mixed = layer.mixer.decode(h, cache.states[li], rows)
            x, h = layer.norm2.add_forward(x, mixed)
            delta = layer.ffn(h)
        cache.lengths_dev += 1
        if delta is None:
            return self.lm_head(self.final_norm(x))
        return self.lm_head(self.final_norm.add_forward(x, delta)[1])

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, cache: HybridCache) -> torch.Tensor:
        """One token per sequence [B] -> logits [B, vocab]; every state and cache advances by one."""
        B = cache.batch
        if tokens.shape != (B,):
            raise ValueError(f"expected [{B}] tokens, got {tuple(tokens.shape)}")
        if max(cache.lengths) >= cache.max_len:
            raise ValueError("the KV cache is full")
        logits = self._decode_body(tokens.to(self.embed.weight.device), cache, max(cache.lengths) + 1)
        cache.lengths = [n + 1 for n in cache.lengths]
        return logits

    @torch.no_grad()
    def capture_decode(self, cache: HybridCache, greedy: bool = True) -> "DecodeGraph":
        """A CUDA graph of one decode step on `cache` (see DecodeGraph)."""
        return DecodeGraph(self, cache, greedy)

    # ------------------------------------------------------------------ reference surface
    def forward(self, input_ids: torch.Tensor, targets: Optional[torch.Tensor] = None
                ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        """Uniform batch [B, T] -> (logits [B, T, vocab], cross-entropy or None) (:97-118)."""
        B, T = input_ids.shape
        dev = self.embed.weight.device
        cache = self.new_cache(B, T)
        cu = [i * T for i in range(B + 1)]
        cu_dev = torch.tensor(cu, device=dev, dtype=torch.int64)
        rows = torch.arange(B, device=dev)
        fresh = torch.ones(B, dtype=torch.bool)
        with torch.no_grad():
            x, delta = self._prefill_body(self.embed(input_ids.to(dev).reshape(-1)), cu, cu_dev, cache, rows, fresh)
            h = self.final_norm(x) if delta is None else self.final_norm.add_forward(x, delta)[1]
            logits = self.lm_head(h).view(B, T, -1)
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.float().view(-1, self.vocab_size), targets.to(dev).view(-1))
        return logits, loss

    @torch.no_grad()
    def prefill_and_init_states(self, prompt_ids: torch.Tensor, max_new_tokens: int = 0
                                ) -> Tuple[torch.Tensor, HybridCache]:
        """[B, T] prompts -> (next-token logits [B, 1, vocab], the cache) (:121-140)."""
        B, T = prompt_ids.shape
        cache = self.new_cache(B, T + max_new_tokens)
        logits = self.prefill(prompt_ids.reshape(-1), [i * T for i in range(B + 1)], cache)
        return logits[:, None, :], cache

    @torch.no_grad()
    def generate(self, prompt_ids: Union[torch.Tensor, List[torch.Tensor]], max_new_tokens: int = 64,
                 temperature: float = 1.0, top_k: Optional[int] = 50, top_p: Optional[float] = 0.95,
                 use_graph: bool = True) -> Union[torch.Tensor, List[torch.Tensor]]:
        """Autoregressive generation with constant-size state per Kernel-DeltaNet layer (:142-197).
        `prompt_ids` is [B, T] (returns [B, T + max_new_tokens]) or a list of 1-D prompts of any
        lengths (returns a list).  temperature <= 0 is greedy; greedy decoding replays a captured
        CUDA graph of the decode step (``use_graph``)."""
        ragged = isinstance(prompt_ids, (list, tuple))
        prompts = list(prompt_ids) if ragged else list(prompt_ids.unbind(0))
        lens = [int(p.numel()) for p in prompts]
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        cache = self.new_cache(len(prompts), max(lens) + max_new_tokens)
        logits = self.prefill(torch.cat([p.reshape(-1) for p in prompts]), cu, cache)
        out = []
        graph = None
        if max_new_tokens > 0:
            out.append(_sample(logits, temperature, top_k, top_p))
            if temperature <= 0.0 and use_graph and max_new_tokens > 2:
                graph = DecodeGraph(self, cache, greedy=True)
                graph.tokens.copy_(out[-1])
        for _ in range(1, max_new_tokens):
            if graph is not None:
                graph.step()  # consumes graph.tokens, leaves the argmax of the new logits there
                out.append(graph.tokens.clone())
            else:
                out.append(_sample(self.decode_step(out[-1], cache), temperature, top_k, top_p))
        gen = torch.stack(out, dim=1) if out else torch.zeros(len(prompts), 0, dtype=torch.int64,
                                                               device=self.embed.weight.device)
        if ragged:
            return [torch.cat([p.to(gen.device), g]) for p, g in zip(prompts, gen.unbind(0))]
        return torch.cat([prompt_ids.to(gen.device), gen], dim=1)


class DecodeGraph:
    """One decode step of `model` on `cache`, captured once as a CUDA graph and replayed per token.

    The eager step launches several hundred small kernels from Python; replaying the graph issues
    them at once.  The anchors attend over the cache's whole key range (max_len) under the length
    mask, since the graph has fixed shapes.  With ``greedy`` the argmax of the logits becomes the
    next step's input inside the graph, so ``step()`` with no argument continues greedy decoding
    without a host round trip; ``step(tokens)`` feeds given tokens instead.  ``logits`` and
    ``tokens`` are the graph's own buffers (overwritten by the next replay).
    """

    def __init__(self, model: KernelDeltaNetLM, cache: HybridCache, greedy: bool = True):
        self.model, self.cache = model, cache
        dev = model.embed.weight.device
        B = cache.batch
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        # warm-up on a scratch cache (library handles, kernel selection); `cache` is not touched
        scratch = model.new_cache(B, 4)
        scratch.lengths_dev = torch.zeros(B, dtype=torch.int64, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                model._decode_body(self.tokens, scratch, scratch.max_len)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        del scratch
        if cache.lengths_dev is None:
            raise ValueError("prefill the cache before capturing its decode step")
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = model._decode_body(self.tokens, cache, cache.max_len)
            if greedy:
                self.tokens.copy_(torch.argmax(self.logits, dim=-1))

    def step(self, tokens: Optional[torch.Tensor] = None) -> torch.Tensor:
        if max(self.cache.lengths) >= self.cache.max_len:
            raise ValueError("the KV cache is full")
        if tokens is not None:
            self.tokens.copy_(tokens)
        self.graph.replay()
        self.cache.lengths = [n + 1 for n in self.cache.lengths]
        return self.logits


def _sample(logits: torch.Tensor, temperature: float, top_k: Optional[int], top_p: Optional[float]) -> torch.Tensor:
    """Greedy for temperature <= 0, else top-k / top-p sampling (models/kernel_deltanet_lm.py:162-186)."""
    if temperature <= 0.0:
        return torch.argmax(logits, dim=-1)
    z = logits.float() / temperature
    if top_k is not None and top_k > 0:
        kth = torch.topk(z, min(top_k, z.shape[-1])).values[:, -1:]
        z = z.masked_fill(z < kth, float("-inf"))
    if top_p is not None and top_p < 1.0:
        sz, si = torch.sort(z, descending=True)
        remove = torch.cumsum(F.softmax(sz, dim=-1), dim=-1) > top_p
        remove[..., 1:] = remove[..., :-1].clone()
        remove[..., 0] = False
        z = z.masked_fill(remove.scatter(1, si, remove), float("-inf"))
    return torch.multinomial(F.softmax(z, dim=-1), 1)[:, 0]


# reference aliases (models/kernel_deltanet_lm.py:200-205)
KernelTTTLM = KernelDeltaNetLM
