"""Structured-FWHT random-feature lift -- drop-in for the reference's kernels/fwht.py.

``FastWalshHadamardProjection`` keeps the reference constructor, buffers and
forward contract (kernels/fwht.py:48-130): the same signs and phase drawn from
``torch.Generator().manual_seed(seed)`` in the same order, the same dense
``Omega`` buffer, and ``forward(x) -> phi`` with

    phi = u / (||u|| + 1e-8),   u = sqrt(2/D) cos(x Omega^T / d_k^(1/4) + b).

The forward runs the libkdn warp-shuffle butterfly kernel (kdn_fwht_lift) on
CUDA tensors; there is no CPU path.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from .. import _lib


def _sylvester(n: int) -> torch.Tensor:
    H = torch.ones(1, 1, dtype=torch.float64)
    while H.shape[0] < n:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    return H


def pack_sign_bits(d: torch.Tensor) -> list[int]:
    """[M, d_k] +-1 -> M integers, bit i set where the sign is -1 (kernels/fwht.py:74-83)."""
    out = []
    for row in d.detach().cpu().tolist():
        v = 0
        for i, s in enumerate(row):
            if s < 0:
                v |= 1 << i
        out.append(v)
    return out


class FastWalshHadamardProjection(nn.Module):
    """Maps d_k -> D through M = D / d_k structured blocks H D3 H D2 H D1 / sqrt(d_k)."""

    def __init__(self, d_k: int = 64, D: int = 512, seed: int = 42):
        super().__init__()
        if D % d_k != 0:
            raise ValueError(f"D ({D}) must be divisible by d_k ({d_k})")
        self.d_k = d_k
        self.D = D
        self.M = D // d_k
        self.seed = seed
        self.scale_norm = 1.0 / math.sqrt(d_k)
        self.tau_star = float(d_k) ** 0.25
        self.tau_star_inv = 1.0 / self.tau_star

        # draw order of kernels/fwht.py:66-86: d1, d2, d3, then the phase b -- always on the host
        # generator, whatever default device the caller constructs modules on
        with torch.device("cpu"):
            self._draw(seed)
        self._proj_cache: dict = {}

    def _draw(self, seed: int) -> None:
        d_k = self.d_k
        D = self.D
        gen = torch.Generator().manual_seed(seed)
        d1 = torch.where(torch.rand(self.M, d_k, generator=gen) > 0.5, 1.0, -1.0)
        d2 = torch.where(torch.rand(self.M, d_k, generator=gen) > 0.5, 1.0, -1.0)
        d3 = torch.where(torch.rand(self.M, d_k, generator=gen) > 0.5, 1.0, -1.0)
        b = torch.rand(D, generator=gen) * (2.0 * math.pi)
        self._set_constants(d1, d2, d3, b)

    @classmethod
    def from_reference(cls, ref) -> "FastWalshHadamardProjection":
        """The projection an existing reference ``FastWalshHadamardProjection`` computes, taken from
        its buffers ``d1, d2, d3`` (signs [M, d_k]) and ``b`` (phase [D]) (kernels/fwht.py:88-92), not
        re-drawn, so any seed (or hand-edited buffers) carries over exactly.  Build it once per
        reference projection and keep it: construction packs the sign bits and forms Omega."""
        d_k, D = int(ref.d_k), int(ref.D)
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self.d_k, self.D, self.M = d_k, D, D // d_k
        self.seed = getattr(ref, "seed", None)
        self.scale_norm = 1.0 / math.sqrt(d_k)
        self.tau_star = float(d_k) ** 0.25
        self.tau_star_inv = 1.0 / self.tau_star
        host = lambda t: torch.as_tensor(t).detach().to("cpu", torch.float32).clone()
        with torch.device("cpu"):
            self._set_constants(host(ref.d1), host(ref.d2), host(ref.d3), host(ref.b))
        self._proj_cache = {}
        return self

    def _set_constants(self, d1: torch.Tensor, d2: torch.Tensor, d3: torch.Tensor, b: torch.Tensor) -> None:
        """Register the sign, phase and dense Omega buffers for signs d1, d2, d3 [M, d_k] and phase b [D]."""
        d_k = self.d_k
        if tuple(d1.shape) != (self.M, d_k) or tuple(b.shape) != (self.D,):
            raise ValueError(f"signs must be [{self.M}, {d_k}] and the phase [{self.D}]")
        self._phase_host = b.clone()  # fp32, not a buffer: dtype casts of the module leave it alone

        bits = [pack_sign_bits(d) for d in (d1, d2, d3)]  # [stage][m]
        as_i64 = lambda u: u - (1 << 64) if u >= (1 << 63) else u  # uint64 bit pattern in an int64
        rad = torch.tensor([[as_i64(bits[s][m]) for s in range(3)] for m in range(self.M)], dtype=torch.int64)
        self._sign_bits = [[bits[s][m] for s in range(3)] for m in range(self.M)]

        self.register_buffer("d1", d1)
        self.register_buffer("d2", d2)
        self.register_buffer("d3", d3)
        self.register_buffer("rademacher_bits", rad, persistent=False)
        self.register_buffer("b", b)

        H = _sylvester(d_k)
        blocks = []
        for m in range(self.M):  # kernels/fwht.py:103-110, exact in float64
            W = H @ torch.diag(d1[m].double())
            W = torch.diag(d2[m].double()) @ W
            W = H @ W
            W = torch.diag(d3[m].double()) @ W
            blocks.append((H @ W) * self.scale_norm)
        self.register_buffer("Omega", torch.cat(blocks, 0).float())

    # ------------------------------------------------------------------ ABI
    def kdn_projection(self, device: torch.device) -> tuple[_lib.KdnProjection, torch.Tensor]:
        """The ``kdn_projection`` struct for ``device`` (and the phase tensor it points to)."""
        device = torch.device(device)
        key = (device.type, device.index)
        phase = self.b
        if phase.device != device or phase.dtype != torch.float32:
            cached = self._proj_cache.get(key)
            if cached is not None and cached[1].data_ptr() != 0:
                phase = cached[1]
            else:
                # from the host copy drawn at construction: a module-wide dtype cast (model.to(bf16))
                # rounds the buffer b, never this copy
                phase = self._phase_host.to(device=device).contiguous()
        s = _lib.KdnProjection()
        s.d_k = self.d_k
        s.D = self.D
        s.tau_inv = self.tau_star_inv
        s.amp = math.sqrt(2.0 / self.D)
        for m in range(self.M):
            for st in range(3):
                s.sign_bits[m][st] = self._sign_bits[m][st]
        s.phase = phase.data_ptr()
        self._proj_cache[key] = (s, phase)
        return s, phase

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """[..., d_k] -> spherically renormalised features [..., D] (kernels/fwht.py:113-130)."""
        if not x.is_cuda:
            raise RuntimeError("kdn_b200 FastWalshHadamardProjection runs on CUDA tensors only")
        if x.shape[-1] != self.d_k:
            raise RuntimeError(f"last dim {x.shape[-1]} != d_k {self.d_k}")
        lib = _lib.load()
        xc = x.contiguous()
        out = torch.empty(*x.shape[:-1], self.D, device=x.device, dtype=x.dtype)
        proj, _phase = self.kdn_projection(x.device)
        n = xc.numel() // self.d_k
        _lib.check(lib.kdn_fwht_lift(xc.data_ptr(), _lib.dtype_code(xc), out.data_ptr(), _lib.dtype_code(out), n,
                                     proj, _lib.stream_handle(x.device)), "kdn_fwht_lift")
        return out
