"""Oracle: affine-semigroup algebra of chunk transitions (test infrastructure only).

The state map of a block of tokens is affine, S_out = S_in A + B, with
A [D, D] and B [dv, D].  Composition follows kernels/blelloch_scan.py:42-56
(and core/associative_algebra.py:45-60):

    (A1, B1) o (A2, B2) = (A1 A2, B1 A2 + B2)

``chunk_block_transition`` builds (A, B) of a token block by running the
chunked oracle twice: once from S=0 (gives B) and once with v=0 from S=I
(gives A, since the map is linear in S when v=0).
"""

from __future__ import annotations

import numpy as np

from .chunked import chunked_deltanet_forward


def compose(t1, t2):
    A1, B1 = t1
    A2, B2 = t2
    return A1 @ A2, B1 @ A2 + B2


def apply_transition(S, t):
    A, B = t
    return S @ A + B


def chunk_block_transition(q, k, v, beta, decay, consts, chunk_size=64, dtype=np.float64):
    N = np.shape(k)[0]
    D = consts.D
    _, B = chunked_deltanet_forward(q, k, v, beta, decay, consts, chunk_size, None, dtype)
    eye = np.broadcast_to(np.eye(D, dtype=dtype), (N, D, D)).copy()
    zeros_v = np.zeros((N, np.shape(k)[1], D), dtype)
    _, A = chunked_deltanet_forward(q, k, zeros_v, beta, decay, consts, chunk_size, eye, dtype)
    return A, B
