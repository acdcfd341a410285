"""Oracle: structured-FWHT random-feature lift (test infrastructure only).

Restates kernels/fwht.py of the reference:

* constants  -- kernels/fwht.py:54-92  (signs d1,d2,d3 drawn in that order by
  ``rand > 0.5`` from a CPU ``torch.Generator`` seeded with ``seed``; phase
  ``b = 2*pi*rand(D)`` drawn afterwards; tau* = d_k ** 0.25)
* dense Omega -- kernels/fwht.py:96-111 (block m = H diag(d3) H diag(d2) H
  diag(d1) / sqrt(d_k), with H the +-1 Sylvester matrix, blocks stacked)
* forward    -- kernels/fwht.py:113-130 (phi = u / (||u|| + 1e-8),
  u = sqrt(2/D) cos(x Omega^T / tau* + b))

The random draws must consume torch's CPU generator in exactly the reference
order, so this module uses torch only for those draws; all arithmetic is numpy.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ProjectionConstants:
    """Signs and phase of one FastWalshHadamardProjection instance."""

    d_k: int
    D: int
    d1: np.ndarray  # [M, d_k] float, entries +-1
    d2: np.ndarray
    d3: np.ndarray
    b: np.ndarray  # [D] float32 phase in [0, 2pi)

    @property
    def M(self) -> int:
        return self.D // self.d_k

    @property
    def tau_star(self) -> float:
        return float(self.d_k) ** 0.25


def make_projection_constants(d_k: int = 64, D: int = 512, seed: int = 42) -> ProjectionConstants:
    """Draw the reference's signs and phase (kernels/fwht.py:66-86)."""
    import torch  # only for the generator stream the reference consumes

    assert D % d_k == 0
    M = D // d_k
    gen = torch.Generator().manual_seed(seed)
    signs = []
    for _ in range(3):  # d1, d2, d3 in this order (fwht.py:69-71)
        r = torch.rand(M, d_k, generator=gen)
        signs.append(np.where(r.numpy() > 0.5, 1.0, -1.0).astype(np.float32))
    b = (torch.rand(D, generator=gen) * (2.0 * math.pi)).numpy().astype(np.float32)  # fwht.py:86
    return ProjectionConstants(d_k, D, signs[0], signs[1], signs[2], b)


def sylvester(n: int) -> np.ndarray:
    """+-1 Sylvester-Hadamard matrix of order n (fwht.py:99-101)."""
    H = np.ones((1, 1))
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]])
    return H


def build_omega(c: ProjectionConstants, dtype=np.float64) -> np.ndarray:
    """Dense Omega [D, d_k] (fwht.py:96-111); exact integers / sqrt(d_k)."""
    H = sylvester(c.d_k)
    blocks = []
    for m in range(c.M):
        W = H @ np.diag(c.d1[m].astype(np.float64))
        W = np.diag(c.d2[m].astype(np.float64)) @ W
        W = H @ W
        W = np.diag(c.d3[m].astype(np.float64)) @ W
        W = (H @ W) / math.sqrt(c.d_k)
        blocks.append(W)
    return np.concatenate(blocks, axis=0).astype(dtype)


def _row_blocks(n: int, parts: int):
    step = max(1, -(-n // parts))
    return [(i, min(n, i + step)) for i in range(0, n, step)]


def lift(x: np.ndarray, c: ProjectionConstants, dtype=np.float64) -> np.ndarray:
    """phi(x) for x [..., d_k] -> [..., D] (fwht.py:123-130).

    The elementwise part runs on a thread pool over row blocks (numpy releases
    the GIL), so the oracle uses all host cores when timed as the CPU baseline.
    """
    import os
    from concurrent.futures import ThreadPoolExecutor

    x = np.asarray(x, dtype=dtype)
    shape = x.shape
    x2 = x.reshape(-1, c.d_k)
    omega_t = np.ascontiguousarray(build_omega(c, dtype).T)
    out = np.empty((x2.shape[0], c.D), dtype)
    tau = dtype(c.tau_star)
    b = c.b.astype(dtype)
    amp = dtype(math.sqrt(2.0 / c.D))
    eps = dtype(1e-8)

    np.matmul(x2, omega_t, out=out)  # one multithreaded BLAS call

    def work(lo_hi):  # elementwise tail per row block (no BLAS inside the pool)
        lo, hi = lo_hi
        z = out[lo:hi]
        z /= tau
        z += b
        np.cos(z, out=z)
        z *= amp
        z /= np.sqrt(np.einsum("ij,ij->i", z, z))[:, None] + eps

    blocks = _row_blocks(x2.shape[0], 4 * (os.cpu_count() or 1))
    if len(blocks) > 1 and x2.shape[0] >= 4096:
        with ThreadPoolExecutor(os.cpu_count()) as ex:
            list(ex.map(work, blocks))
    else:
        for blk in blocks:
            work(blk)
    return out.reshape(*shape[:-1], c.D)
