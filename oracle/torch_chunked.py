"""The reference's CPU PyTorch prefill, restated in torch -- TEST INFRASTRUCTURE / CPU BASELINE ONLY.

This is what the reference runs on a host without a GPU: ``fused_chunked_deltanet_forward``
(kernels/fused_kernel_deltanet.py:31-155) with the dense-Omega lift of
``FastWalshHadamardProjection.forward`` (kernels/fwht.py:113-130).  It does the same torch work per
chunk as the reference -- two lifts, two Gram matmuls, two ``torch.linalg.solve_triangular`` calls
and the readout/update matmuls, in float32 -- so that timing it on the host cores measures the
reference's own CPU path (bench.py's ``cpu_baseline`` and ``--impl reference`` legs).  The numpy
module ``oracle.chunked`` stays the float64 parity checker.

Correspondence (reference line numbers):

  pad T to a multiple of C, beta pad 0, decay pad 1                 :54-62
  g = cumsum(log clamp(decay, 1e-5, 1)); pairwise exp(min(g_i-g_j,0)) :74-77
  per chunk
    phi = u / (|u| + 1e-8), u = sqrt(2/D) cos(x Omega^T / tau* + b)  fwht.py:123-130, used at :95-96
    G_kk = phi_k phi_k^T, G_qk = phi_q phi_k^T                       :99-100
    inv_U = (I + triu(beta_j G_kk, 1))^-1        (solve_triangular)  :102-105
    W~ = diag(beta) inv_U, W_c = diag(beta g_{i->C}) inv_U           :107-111
    V~ = (I + tril(beta_i g_{j->i} G_kk, -1))^-1 (beta V)  (solve)   :113-116
    Y_intra = (G_qk o P_decay o L) V~                                :119-122
    Y_inter = g_inter o (phi_q S^T - (G_qk o L)(S phi_k^T W~)^T)     :125-140
    S <- g_{0->C} (S - S phi_k^T W~ phi_k) + (V^T W_c) phi_k         :143-149

Pinned to the same golden fixtures as ``oracle.chunked`` (tests/test_oracle_golden.py).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np
import torch

from .projection import ProjectionConstants, build_omega


class TorchProjection:
    """The reference's dense lift (kernels/fwht.py:96-130) as float32 torch tensors."""

    def __init__(self, consts: ProjectionConstants):
        self.omega_t = torch.from_numpy(build_omega(consts, np.float32).T.copy())  # [d_k, D]
        self.b = torch.from_numpy(np.asarray(consts.b, np.float32))
        self.tau_inv = 1.0 / consts.tau_star
        self.amp = math.sqrt(2.0 / consts.D)
        self.D = consts.D

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        u = self.amp * torch.cos(torch.matmul(x, self.omega_t) * self.tau_inv + self.b)
        return u / (torch.linalg.vector_norm(u, dim=-1, keepdim=True) + 1e-8)


def chunked_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                    decay: Optional[torch.Tensor], proj: TorchProjection, chunk: int = 64,
                    initial_state: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """q, k [N, T, d_k], v [N, T, d_v], beta/decay [N, T] (float32 CPU tensors) -> (Y [N, T, d_v],
    S [N, d_v, D]).  decay None means 1."""
    N, T, _ = k.shape
    dv = v.shape[-1]
    C = chunk
    if decay is None:
        decay = torch.ones(N, T)
    pad = (-T) % C
    if pad:
        q = torch.nn.functional.pad(q, (0, 0, 0, pad))
        k = torch.nn.functional.pad(k, (0, 0, 0, pad))
        v = torch.nn.functional.pad(v, (0, 0, 0, pad))
        beta = torch.nn.functional.pad(beta, (0, pad), value=0.0)
        decay = torch.nn.functional.pad(decay, (0, pad), value=1.0)
    NC = (T + pad) // C
    qc, kc, vc = (x.reshape(N, NC, C, -1) for x in (q, k, v))
    bc = beta.reshape(N, NC, C)
    g = torch.cumsum(torch.log(decay.reshape(N, NC, C).clamp(1e-5, 1.0)), dim=-1)
    strict_up = torch.triu(torch.ones(C, C), 1)
    strict_lo = torch.tril(torch.ones(C, C), -1)
    eye = torch.eye(C).expand(N, C, C)

    S = torch.zeros(N, dv, proj.D) if initial_state is None else initial_state.clone().float()
    Y = torch.empty(N, NC, C, dv)
    for c in range(NC):
        fk = proj(kc[:, c])
        fq = proj(qc[:, c])
        Gkk = fk @ fk.transpose(-1, -2)
        Gqk = fq @ fk.transpose(-1, -2)
        b = bc[:, c]
        gc = g[:, c]
        inv_u = torch.linalg.solve_triangular(eye + b.unsqueeze(-2) * Gkk * strict_up, eye, upper=True)
        w_tilde = b.unsqueeze(-1) * inv_u
        w_c = (b * torch.exp(gc[:, -1:] - gc)).unsqueeze(-1) * inv_u
        pair = torch.exp(torch.clamp(gc.unsqueeze(-1) - gc.unsqueeze(-2), max=0.0))
        lower = eye + b.unsqueeze(-1) * pair * Gkk * strict_lo
        v_tilde = torch.linalg.solve_triangular(lower, b.unsqueeze(-1) * vc[:, c], upper=False)
        g_shift = torch.nn.functional.pad(gc[:, :-1], (1, 0))
        p_decay = torch.exp(torch.clamp(g_shift.unsqueeze(-1) - gc.unsqueeze(-2), max=0.0))
        y_intra = (Gqk * p_decay * strict_lo) @ v_tilde
        skw = (S @ fk.transpose(-1, -2)) @ w_tilde          # S phi_k^T W~   [N, dv, C]
        corr = (Gqk * strict_lo) @ skw.transpose(-1, -2)     # [N, C, dv]
        qs = fq @ S.transpose(-1, -2)
        g_inter = torch.exp(g_shift).unsqueeze(-1)
        Y[:, c] = y_intra + g_inter * (qs - corr)
        delta = (vc[:, c].transpose(-1, -2) @ w_c) @ fk
        S = torch.exp(gc[:, -1]).view(N, 1, 1) * (S - skw @ fk) + delta
    return Y.reshape(N, NC * C, dv)[:, :T], S
