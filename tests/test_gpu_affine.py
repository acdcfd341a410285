"""GPU parity of the affine-semigroup kernels and the block maps (through the C ABI)
against the oracle and the reference's compose golden vectors.

Tolerance: exact fp32 arithmetic, max relative error <= 1e-4 (bf16 inputs: the
oracle runs on the rounded inputs; the block prefill in bf16 mode keeps the
bf16 bounds 2e-2 on outputs and 1e-2 on the state).
"""

import os

import numpy as np
import pytest
import torch

import oracle
from conftest import fro_rel, rel_err

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
F32_TOL = 1e-4


@pytest.fixture(scope="module")
def kdn():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import kdn_b200

    kdn_b200.load()
    return kdn_b200


@pytest.fixture(scope="module")
def consts():
    return oracle.make_projection_constants(64, 512, 42)


@pytest.fixture(scope="module")
def proj(kdn):
    return kdn.FastWalshHadamardProjection(64, 512, 42).to(DEV)


def dev(a, dtype=torch.float32):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def seq_inputs(seed, N, T, dv=64):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((N, T, 64)); q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((N, T, 64)); k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((N, T, dv))
    beta = 1 / (1 + np.exp(-rng.standard_normal((N, T))))
    decay = 1 / (1 + np.exp(-(rng.standard_normal((N, T)) + 3)))
    S0 = 0.1 * rng.standard_normal((N, dv, 512))
    return q, k, v, beta, decay, S0


def test_compose_matches_reference_golden(kdn, golden_dir):
    g = np.load(os.path.join(golden_dir, "compose.npz"))  # D=8, d_v=4: padded to 16 inside
    A, B = kdn.compose_transitions((dev(g["A1"], torch.float64), dev(g["B1"], torch.float64)),
                                   (dev(g["A2"], torch.float64), dev(g["B2"], torch.float64)))
    assert A.dtype == torch.float64 and A.shape == g["A"].shape and B.shape == g["B"].shape
    assert fro_rel(A.cpu().numpy(), g["A"]) < 1e-6
    assert fro_rel(B.cpu().numpy(), g["B"]) < 1e-6


def test_compose_full_size(kdn):
    rng = np.random.default_rng(1)
    b, D, dv = 3, 512, 64
    A1 = 0.95 * np.eye(D) + 0.05 * rng.standard_normal((b, D, D)) / np.sqrt(D)
    A2 = 0.95 * np.eye(D) + 0.05 * rng.standard_normal((b, D, D)) / np.sqrt(D)
    B1 = rng.standard_normal((b, dv, D))
    B2 = rng.standard_normal((b, dv, D))
    A, B = kdn.compose_transitions((dev(A1), dev(B1)), (dev(A2), dev(B2)))
    Ar, Br = oracle.compose((A1, B1), (A2, B2))
    assert fro_rel(A.cpu().numpy(), Ar) < F32_TOL
    assert rel_err(B.cpu().numpy(), Br) < F32_TOL


def test_compose_is_associative(kdn):
    rng = np.random.default_rng(2)
    b, D, dv = 2, 64, 32
    T = [(dev(rng.standard_normal((b, D, D)) / np.sqrt(D)), dev(rng.standard_normal((b, dv, D)))) for _ in range(3)]
    L = kdn.compose_transitions(kdn.compose_transitions(T[0], T[1]), T[2])
    R = kdn.compose_transitions(T[0], kdn.compose_transitions(T[1], T[2]))
    assert fro_rel(L[0].cpu().numpy(), R[0].cpu().numpy()) < 1e-5
    assert fro_rel(L[1].cpu().numpy(), R[1].cpu().numpy()) < 1e-5


def test_prefix_scans_match_sequential_oracle(kdn):
    # the reference test's shapes (tests/test_blelloch_scan.py:56-100): B=2, N_c=32, d_v=32, D=64
    rng = np.random.default_rng(42)
    b, n_c, dv, D = 2, 32, 32, 64
    trans = [(0.05 * rng.standard_normal((b, D, D)) + 0.95 * np.eye(D), rng.standard_normal((b, dv, D)))
             for _ in range(n_c)]
    S0 = rng.standard_normal((b, dv, D))
    ref, S = [], S0
    for t in trans:
        ref.append(S)
        S = oracle.apply_transition(S, t)
    tt = [(dev(a), dev(c)) for a, c in trans]
    seq = kdn.sequential_prefix_scan(tt, dev(S0))
    tree = kdn.blelloch_prefix_scan(tt, dev(S0))
    assert len(seq) == n_c and len(tree) == n_c
    for c in range(n_c):
        assert fro_rel(seq[c].cpu().numpy(), ref[c]) < F32_TOL
        assert torch.equal(seq[c], tree[c])
    from kdn_b200.kernels.blelloch_scan import prefix_states

    A = torch.stack([a for a, _ in tt])
    B = torch.stack([c for _, c in tt])
    states, final = prefix_states(A, B, None, want_final=True)
    S = np.zeros((b, dv, D))
    for t in trans:
        S = oracle.apply_transition(S, t)
    assert fro_rel(final.cpu().numpy(), S) < F32_TOL
    assert torch.count_nonzero(states[0]) == 0


@pytest.mark.parametrize("chunk", [64, 32])
@pytest.mark.parametrize("in_dtype", [torch.float32, torch.bfloat16])
def test_block_transition_matches_oracle(kdn, proj, consts, chunk, in_dtype):
    N, T = 2, 130
    q, k, v, beta, decay, _ = seq_inputs(5, N, T)
    if in_dtype == torch.bfloat16:
        k, v = (torch.from_numpy(a).bfloat16().double().numpy() for a in (k, v))
    A, B = kdn.chunk_block_transition(dev(k, in_dtype), dev(v, in_dtype), dev(beta), dev(decay), proj, chunk)
    Ar, Br = oracle.chunk_block_transition(q, k, v, beta, decay, consts, chunk)
    assert fro_rel(A.cpu().numpy(), Ar) < F32_TOL
    assert fro_rel(B.cpu().numpy(), Br) < F32_TOL
    # B alone, and A alone, give the same numbers
    _, B2 = kdn.chunk_block_transition(dev(k, in_dtype), dev(v, in_dtype), dev(beta), dev(decay), proj, chunk,
                                       want_A=False)
    A2, none = kdn.chunk_block_transition(dev(k, in_dtype), None, dev(beta), dev(decay), proj, chunk)
    assert none is None and torch.equal(B2, B) and torch.equal(A2, A)


def test_block_transition_empty_block(kdn, proj):
    z = torch.zeros(3, 0, 64, device=DEV)
    A, B = kdn.chunk_block_transition(z, z, torch.zeros(3, 0, device=DEV), None, proj)
    assert torch.equal(A, torch.eye(512, device=DEV).expand(3, -1, -1))
    assert torch.count_nonzero(B) == 0


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_blocks_folded_on_one_device_match_single_pass(kdn, proj, consts, mode):
    """Sequence-parallel arithmetic with the ranks emulated as blocks on one GPU:
    maps per block -> exclusive fold -> block prefill from the entering state."""
    from kdn_b200.kernels.blelloch_scan import prefix_states

    N, T = 2, 300
    cuts = [0, 128, 228, 300]
    q, k, v, beta, decay, S0 = seq_inputs(9, N, T)
    dt = torch.bfloat16 if mode == "bf16" else torch.float32
    if mode == "bf16":
        q, k, v = (torch.from_numpy(a).bfloat16().double().numpy() for a in (q, k, v))
    y_ref, S_ref = oracle.chunked_deltanet_forward(q, k, v, beta, decay, consts, 64, S0)
    blk = lambda a, i, d=torch.float32: dev(a[:, cuts[i]:cuts[i + 1]], d)
    maps = [kdn.chunk_block_transition(blk(k, i, dt), blk(v, i, dt), blk(beta, i), blk(decay, i), proj, 64)
            for i in range(3)]
    A = torch.stack([m[0] for m in maps])
    B = torch.stack([m[1] for m in maps])
    entering, final = prefix_states(A, B, dev(S0), want_final=True)
    assert fro_rel(final.cpu().numpy(), S_ref) < F32_TOL
    ys = []
    for i in range(3):
        y, S = kdn.fused_chunked_deltanet_forward(blk(q, i, dt), blk(k, i, dt), blk(v, i, dt), blk(beta, i),
                                                  blk(decay, i), proj, 64, entering[i], mode=mode)
        ys.append(y.float())
    y = torch.cat(ys, dim=1).cpu().numpy()
    tol_y, tol_s = (2e-2, 1e-2) if mode == "bf16" else (F32_TOL, F32_TOL)
    assert rel_err(y, y_ref) < tol_y
    assert fro_rel(S.cpu().numpy(), S_ref) < tol_s
