"""Oracle: exact gated delta-rule chunked prefill (test infrastructure only).

Restates ``fused_chunked_deltanet_forward`` of the reference,
kernels/fused_kernel_deltanet.py:31-155, batched over the leading (flattened
batch*head) axis with numpy.  Step-by-step correspondence:

  padding to a multiple of C (beta pad 0, decay pad 1)   :54-62
  cumulative log decay, clamped to [1e-5, 1]             :74-77
  pairwise decay exp(min(g_i - g_j, 0))                   :76-77
  per chunk: lift, Gram matrices                          :95-100
    inv_U = (I + triu(beta_j G_kk, 1))^-1                 :102-105
    W~ = diag(beta) inv_U, W_c = diag(beta g_{i->C}) inv_U:107-111
    V~ = (I + tril(beta_i g_{j->i} G_kk, -1))^-1 beta V   :113-116
    Y_intra = (G_qk o P_decay o strict_lower) V~          :119-122
    Y_inter = g_inter o (phi_q S^T - (G_qk o L)(S phi_k^T W~)^T)  :128-140
    S <- g_{0->C} (S - S phi_k^T W~ phi_k) + V^T W_c phi_k         :144-149

``dtype`` selects the arithmetic precision: float64 for the parity checker,
float32 to mirror the reference's own fp32 work when timed as the CPU baseline.
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

from .projection import ProjectionConstants, lift as _lift


def _tri_solve(M: np.ndarray, B: np.ndarray, lower: bool) -> np.ndarray:
    """Solve M X = B for a batch [N, C, C] of unit-diagonal triangular M by
    substitution, vectorised over the batch (the reference calls torch's
    solve_triangular, fused_kernel_deltanet.py:105,116).  numpy-only on purpose:
    mixing scipy's and numpy's bundled BLAS thread pools makes both crawl."""
    C = M.shape[-1]
    X = np.array(B, dtype=M.dtype, copy=True)
    rows = range(C) if lower else range(C - 1, -1, -1)
    for i in rows:
        if lower and i > 0:
            X[:, i] -= np.einsum("nj,njk->nk", M[:, i, :i], X[:, :i])
        elif not lower and i < C - 1:
            X[:, i] -= np.einsum("nj,njk->nk", M[:, i, i + 1:], X[:, i + 1:])
    return X


def chunked_deltanet_forward(
    q: np.ndarray,  # [N, T, d_k]
    k: np.ndarray,  # [N, T, d_k]
    v: np.ndarray,  # [N, T, d_v]
    beta: np.ndarray,  # [N, T]
    decay: Optional[np.ndarray],  # [N, T] or None (== 1)
    consts: ProjectionConstants,
    chunk_size: int = 64,
    initial_state: Optional[np.ndarray] = None,  # [N, d_v, D]
    dtype=np.float64,
    phi_k: Optional[np.ndarray] = None,  # optional pre-lifted features [N, T, D]
    phi_q: Optional[np.ndarray] = None,
) -> Tuple[np.ndarray, np.ndarray]:
    """Returns (Y [N, T, d_v], S [N, d_v, D]) in ``dtype``."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    beta = np.asarray(beta, dtype)
    N, T, _ = k.shape
    dv = v.shape[-1]
    D = consts.D
    C = chunk_size
    if decay is None:
        decay = np.ones((N, T), dtype)
    decay = np.asarray(decay, dtype)

    # fused_kernel_deltanet.py:54-62 -- pad to a multiple of C
    pad = (-T) % C
    if phi_k is None:
        phi_k = _lift(k, consts, dtype)
    if phi_q is None:
        phi_q = _lift(q, consts, dtype)
    phi_k = np.asarray(phi_k, dtype)
    phi_q = np.asarray(phi_q, dtype)
    if pad:
        # the reference pads the raw inputs with zeros and then lifts them; the
        # padded rows have beta = 0 and decay = 1 so they never touch the state,
        # and their outputs are dropped -- lifting zeros is equivalent.
        z = lambda a, w: np.concatenate([a, np.zeros((N, pad, w), dtype)], axis=1)
        phi_k = z(phi_k, D)
        phi_q = z(phi_q, D)
        v = z(v, dv)
        beta = np.concatenate([beta, np.zeros((N, pad), dtype)], axis=1)
        decay = np.concatenate([decay, np.ones((N, pad), dtype)], axis=1)
    Tp = T + pad
    NC = Tp // C

    pk = phi_k.reshape(N, NC, C, D)
    pq = phi_q.reshape(N, NC, C, D)
    vc = v.reshape(N, NC, C, dv)
    bc = beta.reshape(N, NC, C)
    # :74-77 cumulative log decay per chunk
    g = np.cumsum(np.log(np.clip(decay.reshape(N, NC, C), 1e-5, 1.0)), axis=-1)

    upper = np.triu(np.ones((C, C), dtype), 1)
    lower = np.tril(np.ones((C, C), dtype), -1)
    eye = np.eye(C, dtype=dtype)

    S = np.zeros((N, dv, D), dtype) if initial_state is None else np.array(initial_state, dtype)
    Y = np.empty((N, NC, C, dv), dtype)

    for c in range(NC):
        K = pk[:, c]  # [N, C, D]
        Q = pq[:, c]
        V = vc[:, c]  # [N, C, dv]
        b = bc[:, c]  # [N, C]
        gc = g[:, c]  # [N, C]

        G_kk = K @ K.transpose(0, 2, 1)  # :99
        G_qk = Q @ K.transpose(0, 2, 1)  # :100

        # :102-105  (beta scales column j of the strict upper part)
        inv_U = _tri_solve(eye + b[:, None, :] * G_kk * upper, np.broadcast_to(eye, G_kk.shape), lower=False)
        W_tilde = b[:, :, None] * inv_U  # :107
        g_to_end = np.exp(gc[:, -1:] - gc)  # gamma_{i->C}, :110
        W_c = (b * g_to_end)[:, :, None] * inv_U  # :111

        # :113-116  (pairwise decay exp(min(g_i - g_j, 0)) on the strict lower part)
        pair = np.exp(np.minimum(gc[:, :, None] - gc[:, None, :], 0.0))
        L = eye + b[:, :, None] * pair * G_kk * lower
        V_tilde = _tri_solve(L, b[:, :, None] * V, lower=True)

        # :119-122 intra-chunk readout
        g_shift = np.concatenate([np.zeros((N, 1), dtype), gc[:, :-1]], axis=1)
        P_decay = np.exp(np.minimum(g_shift[:, :, None] - gc[:, None, :], 0.0))
        Y_intra = (G_qk * P_decay * lower) @ V_tilde

        # :128-140 inter-chunk readout from the boundary state
        S_K = S @ K.transpose(0, 2, 1)  # [N, dv, C]
        S_K_W = S_K @ W_tilde  # [N, dv, C]
        inter_corr = (G_qk * lower) @ S_K_W.transpose(0, 2, 1)  # [N, C, dv]
        Q_S = Q @ S.transpose(0, 2, 1)  # [N, C, dv]
        g_inter = np.exp(g_shift)[:, :, None]
        Y[:, c] = Y_intra + g_inter * (Q_S - inter_corr)

        # :144-149 boundary state update
        dS = (V.transpose(0, 2, 1) @ W_c) @ K
        S = np.exp(gc[:, -1])[:, None, None] * (S - S_K_W @ K) + dS

    Yo = Y.reshape(N, Tp, dv)[:, :T]
    return Yo, S
