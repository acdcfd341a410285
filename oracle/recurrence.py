"""Oracle: token-by-token delta-rule recurrence and decode step (test infrastructure only).

* ``token_recurrence`` restates ``sequential_deltanet_reference``
  (tests/test_fused_kernel.py:33-67) with an optional initial state:
      y_t = S_{t-1} phi_q_t
      S_t = lambda_t (S_{t-1} - beta_t (S_{t-1} phi_k_t) phi_k_t^T) + beta_t v_t phi_k_t^T
* ``decode_step`` is one step of the module decode loop
  (kernels/kernel_deltanet_fused.py:288-300): read out BEFORE the update.
* ``decode_step_post`` is the benchmark variant that reads out AFTER the
  update (benchmarks/run_full_batch_decoding.py:27-55).
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

from .projection import ProjectionConstants, lift as _lift


def token_recurrence(
    q, k, v, beta, decay, consts: ProjectionConstants,
    initial_state: Optional[np.ndarray] = None, dtype=np.float64,
) -> Tuple[np.ndarray, np.ndarray]:
    """q,k [N,T,d_k], v [N,T,dv], beta/decay [N,T] -> (Y [N,T,dv], S [N,dv,D])."""
    pk = _lift(np.asarray(k, dtype), consts, dtype)
    pq = _lift(np.asarray(q, dtype), consts, dtype)
    v = np.asarray(v, dtype)
    beta = np.asarray(beta, dtype)
    N, T, dv = v.shape
    decay = np.ones((N, T), dtype) if decay is None else np.asarray(decay, dtype)
    S = np.zeros((N, dv, consts.D), dtype) if initial_state is None else np.array(initial_state, dtype)
    Y = np.empty((N, T, dv), dtype)
    for t in range(T):
        Y[:, t] = np.einsum("nvd,nd->nv", S, pq[:, t])  # test_fused_kernel.py:61
        s_phi = np.einsum("nvd,nd->nv", S, pk[:, t])  # :64
        lt = decay[:, t][:, None, None]
        bt = beta[:, t][:, None, None]
        S = lt * (S - bt * s_phi[:, :, None] * pk[:, t][:, None, :]) + bt * v[:, t][:, :, None] * pk[:, t][:, None, :]
    return Y, S


def _step(S, phi_k, phi_q, v, beta, decay, post: bool):
    s_phi = np.einsum("...vd,...d->...v", S, phi_k)
    y_pre = np.einsum("...vd,...d->...v", S, phi_q)
    lt = decay[..., None, None]
    bt = beta[..., None, None]
    S_new = lt * (S - bt * s_phi[..., :, None] * phi_k[..., None, :]) + bt * v[..., :, None] * phi_k[..., None, :]
    y = np.einsum("...vd,...d->...v", S_new, phi_q) if post else y_pre
    return y, S_new


def decode_step(S, q, k, v, beta, decay, consts: ProjectionConstants, dtype=np.float64):
    """One decode token per (stream, head): S [..., dv, D]; q,k [..., d_k]; v [..., dv].

    Readout before the update, kernels/kernel_deltanet_fused.py:290 then :299-300.
    """
    S = np.asarray(S, dtype)
    pk = _lift(np.asarray(k, dtype), consts, dtype)
    pq = _lift(np.asarray(q, dtype), consts, dtype)
    decay = np.ones(np.shape(beta), dtype) if decay is None else np.asarray(decay, dtype)
    return _step(S, pk, pq, np.asarray(v, dtype), np.asarray(beta, dtype), decay, post=False)


def decode_step_post(S, q, k, v, beta, decay, consts: ProjectionConstants, dtype=np.float64):
    """Readout after the update (benchmarks/run_full_batch_decoding.py:43-54)."""
    S = np.asarray(S, dtype)
    pk = _lift(np.asarray(k, dtype), consts, dtype)
    pq = _lift(np.asarray(q, dtype), consts, dtype)
    decay = np.ones(np.shape(beta), dtype) if decay is None else np.asarray(decay, dtype)
    return _step(S, pk, pq, np.asarray(v, dtype), np.asarray(beta, dtype), decay, post=True)
