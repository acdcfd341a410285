"""Backward of the chunked prefill (row f3).

CPU: the float64 oracle backward against the reference's own gradients (its autograd
Function, recompute + autograd.grad, kernels/fused_kernel_deltanet.py:158-179, fixtures
tests/golden/backward_*.npz) and, for the initial/final-state paths the reference does not
differentiate, against central finite differences of the oracle forward; C-ABI checks.
GPU: libkdn's backward against the same fixtures and against the oracle (initial state,
final-state adjoint, decays outside the clamp range, chunk 32 with d_v 128, bf16 inputs,
T = 1), through the C-ABI wrapper and through autograd.  Tolerance: max |error| <= 1e-4 of
the largest gradient entry (fp32 vs fp32 autograd / float64).
"""

import os

import numpy as np
import pytest
import torch

import oracle
from oracle.backward import chunked_deltanet_backward as oracle_backward

GOLD = os.path.join(os.path.dirname(__file__), "golden")
CASES = ("backward_t130_gated", "backward_t63_n2", "backward_c32_dv128_gated")
KEYS = ("dq", "dk", "dv", "dbeta", "ddecay")


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_gradients(name):
    z = np.load(os.path.join(GOLD, f"{name}.npz"))
    r = oracle_backward(z["q"], z["k"], z["v"], z["beta"], z["decay"], z["dY"], oracle.make_projection_constants())
    for key in KEYS:
        assert _rel(r[key], z[key]) <= 1e-5, key


def test_oracle_state_gradients_by_finite_differences():
    """L = <Y, dY> + <S_T, dS_T>: directional derivatives along random directions."""
    rng = np.random.default_rng(3)
    c = oracle.make_projection_constants()
    N, T, dv = 1, 9, 16
    q = rng.standard_normal((N, T, 64)); q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((N, T, 64)); k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((N, T, dv))
    beta = 1 / (1 + np.exp(-rng.standard_normal((N, T))))
    decay = 1 / (1 + np.exp(-(rng.standard_normal((N, T)) + 2)))
    S0 = 0.3 * rng.standard_normal((N, dv, 512))
    dY = rng.standard_normal((N, T, dv))
    dS = rng.standard_normal((N, dv, 512))

    def loss(q_, k_, v_, b_, d_, s_):
        Y, S = oracle.chunked_deltanet_forward(q_, k_, v_, b_, d_, c, 4, s_)
        return float((Y * dY).sum() + (S * dS).sum())

    g = oracle_backward(q, k, v, beta, decay, dY, c, initial_state=S0, dS_final=dS)
    base = [q, k, v, beta, decay, S0]
    grads = [g["dq"], g["dk"], g["dv"], g["dbeta"], g["ddecay"], g["dS0"]]
    h = 1e-5
    for idx in range(6):
        d = rng.standard_normal(base[idx].shape)
        plus = list(base); plus[idx] = base[idx] + h * d
        minus = list(base); minus[idx] = base[idx] - h * d
        fd = (loss(*plus) - loss(*minus)) / (2 * h)
        an = float((grads[idx] * d).sum())
        assert abs(fd - an) <= 1e-6 * max(1.0, abs(an)), (idx, fd, an)


def test_backward_argument_checks(lib):
    from kdn_b200.kernels.fwht import FastWalshHadamardProjection

    proj, _ = FastWalshHadamardProjection().kdn_projection(torch.device("cpu"))
    P = 4096
    args = lambda **kw: [kw.get(n, d) for n, d in (
        ("q", P), ("k", P), ("v", P), ("idt", 0), ("beta", P), ("decay", None), ("gdt", 0), ("S0", None), ("dy", P),
        ("ydt", 0), ("dSf", None), ("dq", P), ("dk", P), ("dv_", P), ("db", P), ("dd", None), ("dS0", None),
        ("N", 1), ("T", 8), ("dv", 64), ("C", 64))] + [proj, P, 1 << 30, None]
    assert lib.kdn_chunked_prefill_backward(*args(dv=256)) == 2     # d_v above 128
    assert lib.kdn_chunked_prefill_backward(*args(C=16)) == 2       # chunk 16
    assert lib.kdn_chunked_prefill_backward(*args(dq=None)) == 1    # missing gradient output
    assert lib.kdn_chunked_prefill_backward(*args(N=0)) == 1
    assert lib.kdn_chunked_prefill_backward(*(args()[:-4] + [proj, P, 16, None])) == 4  # workspace too small
    assert lib.kdn_chunked_prefill_backward_workspace_size(2, 100, 64, 64, proj) > 0


# ---------------------------------------------------------------------------- GPU
def _cuda(a, dtype=torch.float32):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_libkdn_backward_matches_reference_gradients(name):
    from kdn_b200 import FastWalshHadamardProjection, chunked_deltanet_backward

    z = np.load(os.path.join(GOLD, f"{name}.npz"))
    C = int(z["meta"][5])
    g = chunked_deltanet_backward(_cuda(z["q"]), _cuda(z["k"]), _cuda(z["v"]), _cuda(z["beta"]), _cuda(z["decay"]),
                                  _cuda(z["dY"]), FastWalshHadamardProjection().cuda(), C)
    for key in KEYS:
        assert _rel(g[key].cpu().numpy(), z[key]) <= 1e-4, key


def _inputs(seed, N, T, dv, extreme=False):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((N, T, 64)); q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((N, T, 64)); k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((N, T, dv))
    beta = 1 / (1 + np.exp(-rng.standard_normal((N, T))))
    decay = 1 / (1 + np.exp(-(rng.standard_normal((N, T)) + 3)))
    if extreme:  # entries the clamp of the reference cuts (no gradient) and exact ones
        decay[:, ::7] = 1.0
        decay[:, 3::11] = 1.5
        decay[:, 5::13] = 1e-7
    S0 = 0.1 * rng.standard_normal((N, dv, 512))
    dY = rng.standard_normal((N, T, dv))
    dS = 0.1 * rng.standard_normal((N, dv, 512))
    return q, k, v, beta, decay, S0, dY, dS


@pytest.mark.gpu
@pytest.mark.parametrize("N,T,dv,C,extreme", [(3, 200, 64, 64, True), (1, 77, 128, 32, False), (2, 1, 64, 64, False)])
def test_libkdn_backward_matches_oracle_with_states(N, T, dv, C, extreme):
    from kdn_b200 import FastWalshHadamardProjection, chunked_deltanet_backward

    q, k, v, beta, decay, S0, dY, dS = _inputs(N + T, N, T, dv, extreme)
    r = oracle_backward(q, k, v, beta, decay, dY, oracle.make_projection_constants(), S0, dS)
    g = chunked_deltanet_backward(_cuda(q), _cuda(k), _cuda(v), _cuda(beta), _cuda(decay), _cuda(dY),
                                  FastWalshHadamardProjection().cuda(), C, _cuda(S0), _cuda(dS))
    for key, ref in (("dq", r["dq"]), ("dk", r["dk"]), ("dv", r["dv"]), ("dbeta", r["dbeta"]),
                     ("ddecay", r["ddecay"]), ("d_initial_state", r["dS0"])):
        assert _rel(g[key].cpu().numpy(), ref) <= 1e-4, key
    if extreme:
        dd = g["ddecay"].cpu().numpy()
        assert np.all(dd[:, 3::11] == 0) and np.all(dd[:, 5::13] == 0)


@pytest.mark.gpu
def test_libkdn_backward_bf16_inputs():
    from kdn_b200 import FastWalshHadamardProjection, chunked_deltanet_backward

    q, k, v, beta, decay, S0, dY, dS = _inputs(5, 2, 150, 64)
    qb, kb, vb = (torch.from_numpy(a).bfloat16() for a in (q, k, v))
    r = oracle_backward(qb.double().numpy(), kb.double().numpy(), vb.double().numpy(), beta, decay, dY,
                        oracle.make_projection_constants(), None, None)
    g = chunked_deltanet_backward(qb.cuda(), kb.cuda(), vb.cuda(), _cuda(beta), _cuda(decay), _cuda(dY),
                                  FastWalshHadamardProjection().cuda(), 64)
    for key in KEYS:
        assert _rel(g[key].cpu().numpy(), r[key]) <= 1e-4, key


@pytest.mark.gpu
def test_autograd_through_both_surfaces():
    from kdn_b200 import FastWalshHadamardProjection, fused_chunked_deltanet_forward
    from kdn_b200.kernels.fused_kernel_deltanet import FusedKernelDeltaNetFunction

    q, k, v, beta, decay, S0, dY, dS = _inputs(9, 2, 100, 64)
    proj = FastWalshHadamardProjection().cuda()
    ins = [_cuda(a).requires_grad_(True) for a in (q, k, v, beta, decay, S0)]
    Y, S = fused_chunked_deltanet_forward(*ins[:5], proj, 64, ins[5], mode="fp32")
    ((Y * _cuda(dY)).sum() + (S * _cuda(dS)).sum()).backward()
    r = oracle_backward(q, k, v, beta, decay, dY, oracle.make_projection_constants(), S0, dS)
    for t, key in zip(ins, ("dq", "dk", "dv", "dbeta", "ddecay", "dS0")):
        assert _rel(t.grad.cpu().numpy(), r[key]) <= 1e-4, key
    # the reference-named Function: Y only, no initial state
    z = np.load(os.path.join(GOLD, "backward_t130_gated.npz"))
    ins = [_cuda(z[n]).requires_grad_(True) for n in ("q", "k", "v", "beta", "decay")]
    FusedKernelDeltaNetFunction.apply(*ins, proj, 64).backward(_cuda(z["dY"]))
    for t, key in zip(ins, KEYS):
        assert _rel(t.grad.cpu().numpy(), z[key]) <= 1e-4, key


@pytest.mark.gpu
def test_empty_sequence_passes_the_state_gradient():
    from kdn_b200 import _lib
    from kdn_b200.kernels.fwht import FastWalshHadamardProjection

    lib = _lib.load()
    proj, _ = FastWalshHadamardProjection().cuda().kdn_projection(torch.device("cuda"))
    dS = torch.randn(2, 64, 512, device="cuda")
    dS0 = torch.full_like(dS, 7.0)
    rc = lib.kdn_chunked_prefill_backward(None, None, None, 0, None, None, 0, None, None, 0, dS.data_ptr(), None,
                                          None, None, None, None, dS0.data_ptr(), 2, 0, 64, 64, proj, None, 0,
                                          _lib.stream_handle(dS.device))
    torch.cuda.synchronize()
    assert rc == 0 and torch.equal(dS0, dS)
