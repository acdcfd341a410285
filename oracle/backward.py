"""Oracle: gradients of the chunked delta-rule prefill (TEST INFRASTRUCTURE ONLY).

The reference's backward (kernels/fused_kernel_deltanet.py:158-179) recomputes the forward
under autograd and returns d(Y . dY)/d(q, k, v, beta, decay).  Its forward is the exact
gated delta rule (kernels/fused_kernel_deltanet.py:31-155, restated by
``oracle.chunked``), so its gradient is the gradient of the token recurrence

    u_t = S_{t-1} phik_t,   y_t = S_{t-1} phiq_t,
    S_t = lam_t S_{t-1} + beta_t (v_t - lam_t u_t) phik_t^T,   lam_t = clamp(decay_t, 1e-5, 1)

(the clamp of :74 passes the gradient where 1e-5 <= decay <= 1, zero elsewhere; its other
clamps act on masked entries only), followed by the lift phi(x) = u / (||u|| + 1e-8),
u = sqrt(2/D) cos(x Omega^T / tau + b) (kernels/fwht.py:123-130).  This module runs that
recurrence backwards in float64, one token at a time, and also returns the gradient of an
optional initial state and accepts one for the final state (the reference's autograd
returns neither; the chunked forward accepts an initial state, :39).
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np

from .projection import ProjectionConstants, build_omega, lift


def lift_backward(x, dphi, c: ProjectionConstants, dtype=np.float64):
    """x [..., d_k], dphi [..., D] -> d(phi . dphi)/dx [..., d_k]."""
    x = np.asarray(x, dtype)
    shape = x.shape
    x2 = x.reshape(-1, c.d_k)
    g = np.asarray(dphi, dtype).reshape(-1, c.D)
    omega = build_omega(c, dtype)  # [D, d_k]
    tau_inv = 1.0 / float(c.tau_star)
    amp = math.sqrt(2.0 / c.D)
    z = x2 @ omega.T * tau_inv + c.b.astype(dtype)
    u = amp * np.cos(z)
    n = np.sqrt(np.einsum("ij,ij->i", u, u))[:, None]
    e = n + 1e-8
    du = g / e - u * np.einsum("ij,ij->i", u, g)[:, None] / (n * e * e)
    dz = -du * amp * np.sin(z)
    return ((dz @ omega) * tau_inv).reshape(shape)


def chunked_deltanet_backward(q, k, v, beta, decay, dY, c: ProjectionConstants,
                              initial_state: Optional[np.ndarray] = None, dS_final: Optional[np.ndarray] = None,
                              dtype=np.float64):
    """q, k [N, T, d_k], v / dY [N, T, dv], beta / decay [N, T] (decay None == 1).

    Returns dict(dq, dk, dv, dbeta, ddecay (None when decay is None), dS0)."""
    q, k, v, beta, dY = (np.asarray(a, dtype) for a in (q, k, v, beta, dY))
    N, T, dv = v.shape
    D = c.D
    lam_raw = np.ones((N, T), dtype) if decay is None else np.asarray(decay, dtype)
    lam = np.clip(lam_raw, 1e-5, 1.0)
    pass_mask = ((lam_raw >= 1e-5) & (lam_raw <= 1.0)).astype(dtype)
    pk = lift(k, c, dtype)
    pq = lift(q, c, dtype)
    S = np.zeros((N, dv, D), dtype) if initial_state is None else np.array(initial_state, dtype)
    prev = np.empty((T, N, dv, D), dtype)
    for t in range(T):
        prev[t] = S
        u = np.einsum("nvd,nd->nv", S, pk[:, t])
        S = lam[:, t, None, None] * S + (beta[:, t, None] * (v[:, t] - lam[:, t, None] * u))[:, :, None] * \
            pk[:, t, None, :]
    dS = np.zeros((N, dv, D), dtype) if dS_final is None else np.array(dS_final, dtype)
    dpk = np.zeros_like(pk)
    dpq = np.zeros_like(pq)
    dvv = np.zeros_like(v)
    db = np.zeros((N, T), dtype)
    dl = np.zeros((N, T), dtype)
    for t in range(T - 1, -1, -1):
        Sp = prev[t]
        kt, qt = pk[:, t], pq[:, t]
        lt, bt = lam[:, t], beta[:, t]
        u = np.einsum("nvd,nd->nv", Sp, kt)
        g = np.einsum("nvd,nd->nv", dS, kt)
        r = v[:, t] - lt[:, None] * u
        dpq[:, t] = np.einsum("nvd,nv->nd", Sp, dY[:, t])
        dvv[:, t] = bt[:, None] * g
        db[:, t] = np.einsum("nv,nv->n", g, r)
        dl[:, t] = np.einsum("nvd,nvd->n", dS, Sp) - bt * np.einsum("nv,nv->n", g, u)
        dpk[:, t] = bt[:, None] * np.einsum("nvd,nv->nd", dS, r) - (lt * bt)[:, None] * np.einsum("nvd,nv->nd", Sp, g)
        dS = lt[:, None, None] * dS - (lt * bt)[:, None, None] * g[:, :, None] * kt[:, None, :] + \
            dY[:, t, :, None] * qt[:, None, :]
    return {"dq": lift_backward(q, dpq, c, dtype), "dk": lift_backward(k, dpk, c, dtype), "dv": dvv, "dbeta": db,
            "ddecay": None if decay is None else dl * pass_mask, "dS0": dS}
