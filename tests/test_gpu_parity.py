"""GPU parity of libkdn (through the C ABI) against the CPU oracle and the
reference's golden vectors.

Tolerances (stated by the build contract):
  fp32 mode : max relative error <= 1e-4 (outputs per row and state)
  bf16 mode : outputs <= 2e-2, final state <= 1e-2, against the oracle run on
              the bf16-rounded inputs
"""

import os

import numpy as np
import pytest
import torch

import oracle
from conftest import fro_rel, rel_err

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_Y_TOL = 2e-2
BF16_S_TOL = 1e-2

DEV = "cuda:0"


@pytest.fixture(scope="module")
def kdn():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import kdn_b200

    kdn_b200.load()
    return kdn_b200


@pytest.fixture(scope="module")
def proj(kdn):
    return kdn.FastWalshHadamardProjection(64, 512, 42).to(DEV)


@pytest.fixture(scope="module")
def consts():
    return oracle.make_projection_constants(64, 512, 42)


def make_inputs(seed, N, T, dv=64, gated=False, init=False, D=512):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((N, T, 64)); q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((N, T, 64)); k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((N, T, dv))
    beta = 1 / (1 + np.exp(-rng.standard_normal((N, T))))
    decay = 1 / (1 + np.exp(-(rng.standard_normal((N, T)) + 3))) if gated else None
    S0 = 0.1 * rng.standard_normal((N, dv, D)) if init else None
    f = lambda a: None if a is None else a.astype(np.float32)
    return f(q), f(k), f(v), f(beta), f(decay), f(S0)


def to_dev(a, dtype=torch.float32):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def bf16_round(a):
    return None if a is None else torch.from_numpy(a).bfloat16().float().numpy()


# ------------------------------------------------------------------ lift
@pytest.mark.parametrize("seed", [42, 7])
def test_lift_matches_reference_golden(kdn, golden_dir, seed):
    g = np.load(os.path.join(golden_dir, f"lift_seed{seed}.npz"))
    p = kdn.FastWalshHadamardProjection(64, 512, seed).to(DEV)
    phi = p(to_dev(g["x"])).cpu().numpy()
    assert rel_err(phi, g["phi"]) < 2e-5


def test_lift_many_vectors_and_bf16(proj, consts):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((3, 1000, 64)).astype(np.float32)
    x /= np.linalg.norm(x, axis=-1, keepdims=True)
    ref = oracle.lift(x, consts)
    got = proj(to_dev(x)).cpu().numpy()
    assert got.shape == (3, 1000, 512)
    assert rel_err(got, ref) < 2e-5
    xb = to_dev(x, torch.bfloat16)
    got_b = proj(xb).float().cpu().numpy()
    ref_b = oracle.lift(xb.float().cpu().numpy(), consts)
    assert rel_err(got_b, ref_b) < 1e-2  # bf16 output rounding
    np.testing.assert_allclose(np.linalg.norm(got, axis=-1), 1.0, atol=1e-5)


@pytest.mark.parametrize("D,seed", [(512, 42), (128, 11)])
@pytest.mark.parametrize("path", ["", "pair"])
def test_lift_paths_and_mixed_dtypes(kdn, monkeypatch, D, seed, path):
    """kdn_fwht_lift through the C ABI on every input/output dtype pair, with a ragged last tile:
    bf16 inputs at D = 512 with a bf16-exact Omega (seed 42) take the tensor-core kernel unless
    KDN_LIFT_PATH=pair; the rest take the lane-pair kernel; rows only 8-byte aligned take the
    one-warp kernel.  All against the oracle."""
    from kdn_b200 import _lib
    from kdn_b200.serving.vllm_kernel_deltanet_op import device_error

    monkeypatch.setenv("KDN_LIFT_PATH", path)
    lib = _lib.load()
    p = kdn.FastWalshHadamardProjection(64, D, seed).to(DEV)
    c = oracle.make_projection_constants(64, D, seed)
    pstruct, _phase = p.kdn_projection(torch.device(DEV))
    rng = np.random.default_rng(4)
    n = 128 * 9 + 37  # also 16 * 74 + 5: a ragged last group for both kernels
    x = rng.standard_normal((n, 64)).astype(np.float32)
    x /= np.linalg.norm(x, axis=-1, keepdims=True)
    for xd in (torch.float32, torch.bfloat16):
        xt = to_dev(x, xd)
        ref = oracle.lift(xt.float().cpu().numpy(), c)
        for od in (torch.float32, torch.bfloat16):
            out = torch.full((n, D), float("nan"), device=DEV, dtype=od)
            rc = lib.kdn_fwht_lift(xt.data_ptr(), _lib.dtype_code(xt), out.data_ptr(), _lib.dtype_code(out), n,
                                   pstruct, None)
            torch.cuda.synchronize()
            assert rc == 0
            tol = 2e-5 if od == torch.float32 else 1e-2
            assert rel_err(out.float().cpu().numpy(), ref) < tol, (xd, od)
    assert device_error(DEV) == 0
    # 8-byte aligned (not 16): input rows start 2 floats into a padded buffer, output 2 floats in
    xb = torch.zeros(n * 64 + 2, device=DEV)
    xb[2:] = to_dev(x).reshape(-1)
    ob = torch.full((n * D + 2,), float("nan"), device=DEV)
    assert lib.kdn_fwht_lift(xb.data_ptr() + 8, 0, ob.data_ptr() + 8, 0, n, pstruct, None) == 0
    torch.cuda.synchronize()
    assert rel_err(ob[2:].view(n, D).cpu().numpy(), oracle.lift(x, c)) < 2e-5


def test_lift_tensor_core_path_agrees(kdn, proj, monkeypatch):
    """The default projection's Omega is bf16-exact, so bf16 inputs take the tensor-core lift: on a batch
    of several tiles per CTA it agrees with the lane-pair kernel element by element to within one bf16 ulp."""
    g = torch.Generator(device=DEV).manual_seed(9)
    xb = torch.nn.functional.normalize(torch.randn(148 * 128 * 3 + 77, 64, generator=g, device=DEV), dim=-1).bfloat16()
    monkeypatch.setenv("KDN_LIFT_PATH", "")
    a = proj(xb).float()
    monkeypatch.setenv("KDN_LIFT_PATH", "pair")
    b = proj(xb).float()
    # at most one bf16 ulp apart (the two kernels round different fp32 values; ulp <= 2^-7 |x|)
    assert bool(((a - b).abs() <= 2.0 ** -7 * torch.maximum(a.abs(), b.abs()) + 1e-6).all())
    np.testing.assert_allclose(a.norm(dim=-1).cpu().numpy(), 1.0, atol=1e-2)


# --------------------------------------------------------------- prefill
GOLDEN_PREFILL = ["prefill_t130_gated_s0", "prefill_t63", "prefill_t64", "prefill_t1",
                  "prefill_c32_dv128_gated", "prefill_t256_c64"]


@pytest.mark.parametrize("name", GOLDEN_PREFILL)
def test_prefill_fp32_matches_reference_golden(kdn, proj, golden_dir, name):
    g = np.load(os.path.join(golden_dir, name + ".npz"))
    seed, N, T, d_k, dv, C, gated, init = [int(x) for x in g["meta"]]
    Y, S = kdn.fused_chunked_deltanet_forward(
        to_dev(g["q"]), to_dev(g["k"]), to_dev(g["v"]), to_dev(g["beta"]), to_dev(g["decay"]), proj, C,
        to_dev(g["S0"]) if init else None, mode="fp32")
    torch.cuda.synchronize()
    assert rel_err(Y.cpu().numpy(), g["Y"]) < F32_TOL
    assert fro_rel(S.cpu().numpy(), g["S"]) < F32_TOL


CASES = [
    # (seed, N, T, dv, C, gated, init)
    (10, 3, 1, 64, 64, False, False),
    (11, 2, 63, 64, 64, True, True),
    (12, 2, 64, 64, 64, False, True),
    (13, 2, 65, 64, 64, True, False),
    (14, 2, 130, 64, 64, False, False),
    (15, 1, 200, 32, 32, True, True),
    (16, 4, 517, 64, 64, True, False),
    (17, 1, 96, 128, 32, False, True),
]


@pytest.mark.parametrize("case", CASES)
def test_prefill_fp32_vs_oracle(kdn, proj, consts, case):
    seed, N, T, dv, C, gated, init = case
    q, k, v, beta, decay, S0 = make_inputs(seed, N, T, dv, gated, init)
    Y, S = kdn.fused_chunked_deltanet_forward(to_dev(q), to_dev(k), to_dev(v), to_dev(beta), to_dev(decay), proj, C,
                                              to_dev(S0), mode="fp32")
    Yr, Sr = oracle.chunked_deltanet_forward(q, k, v, beta, decay, consts, C, S0)
    assert rel_err(Y.cpu().numpy(), Yr) < F32_TOL
    assert fro_rel(S.cpu().numpy(), Sr) < F32_TOL


@pytest.mark.parametrize("case", [(20, 2, 130, 64, 64, True, True), (21, 4, 1000, 64, 64, False, False),
                                  (22, 1, 257, 64, 32, True, False)])
def test_prefill_bf16_vs_oracle(kdn, proj, consts, case):
    seed, N, T, dv, C, gated, init = case
    q, k, v, beta, decay, S0 = make_inputs(seed, N, T, dv, gated, init)
    qb, kb, vb = (to_dev(a, torch.bfloat16) for a in (q, k, v))
    Y, S = kdn.fused_chunked_deltanet_forward(qb, kb, vb, to_dev(beta), to_dev(decay), proj, C, to_dev(S0),
                                              mode="bf16")
    assert Y.dtype == torch.bfloat16 and S.dtype == torch.float32
    Yr, Sr = oracle.chunked_deltanet_forward(bf16_round(q), bf16_round(k), bf16_round(v), beta, decay, consts, C,
                                             S0)
    assert rel_err(Y.float().cpu().numpy(), Yr) < BF16_Y_TOL
    assert fro_rel(S.cpu().numpy(), Sr) < BF16_S_TOL


def test_prefill_resume_equals_single_pass(kdn, proj):
    q, k, v, beta, decay, _ = make_inputs(30, 2, 300, 64, True)
    dq, dk, dv_, db, dd = (to_dev(a) for a in (q, k, v, beta, decay))
    Y, S = kdn.fused_chunked_deltanet_forward(dq, dk, dv_, db, dd, proj, 64, mode="fp32")
    Y1, S1 = kdn.fused_chunked_deltanet_forward(dq[:, :130], dk[:, :130], dv_[:, :130], db[:, :130], dd[:, :130],
                                                proj, 64, mode="fp32")
    Y2, S2 = kdn.fused_chunked_deltanet_forward(dq[:, 130:], dk[:, 130:], dv_[:, 130:], db[:, 130:], dd[:, 130:],
                                                proj, 64, S1, mode="fp32")
    assert rel_err(torch.cat([Y1, Y2], 1).cpu().numpy(), Y.cpu().numpy()) < 1e-5
    assert fro_rel(S2.cpu().numpy(), S.cpu().numpy()) < 1e-5


def test_prefill_equals_token_recurrence(kdn, proj, consts):
    q, k, v, beta, decay, S0 = make_inputs(31, 2, 80, 64, True, True)
    Y, S = kdn.fused_chunked_deltanet_forward(to_dev(q), to_dev(k), to_dev(v), to_dev(beta), to_dev(decay), proj, 32,
                                              to_dev(S0), mode="fp32")
    Yr, Sr = oracle.token_recurrence(q, k, v, beta, decay, consts, S0)
    assert rel_err(Y.cpu().numpy(), Yr) < F32_TOL
    assert fro_rel(S.cpu().numpy(), Sr) < F32_TOL


def test_prefill_empty_sequence(kdn, proj):
    S0 = torch.randn(2, 64, 512, device=DEV)
    x = torch.empty(2, 0, 64, device=DEV)
    Y, S = kdn.fused_chunked_deltanet_forward(x, x, x, torch.empty(2, 0, device=DEV), None, proj, 64, S0)
    torch.cuda.synchronize()
    assert Y.shape == (2, 0, 64)
    assert torch.equal(S, S0)


def test_layer_surface(kdn, consts):
    B, H, T = 2, 3, 70
    layer = kdn.KernelDeltaNetLayer(num_heads=H, mode="fp32").to(DEV)
    q, k, v, beta, decay, S0 = make_inputs(40, B * H, T, 64, True, True)
    r = lambda a, w: to_dev(a.reshape(B, H, T, w))
    y, S = layer(r(q, 64), r(k, 64), r(v, 64), to_dev(beta.reshape(B, H, T)),
                 state=to_dev(S0.reshape(B, H, 64, 512)), decay=to_dev(decay.reshape(B, H, T)))
    assert y.shape == (B, H, T, 64) and S.shape == (B, H, 64, 512)
    Yr, Sr = oracle.chunked_deltanet_forward(q, k, v, beta, decay, consts, 64, S0)
    assert rel_err(y.reshape(B * H, T, 64).cpu().numpy(), Yr) < F32_TOL
    assert fro_rel(S.reshape(B * H, 64, 512).cpu().numpy(), Sr) < F32_TOL
    assert kdn.KernelTTTLayer is kdn.KernelDeltaNetLayer


# ----------------------------------------------------------------- decode
def _decode_inputs(seed, ntok, H, slots):
    rng = np.random.default_rng(seed)
    S = (0.02 * rng.standard_normal((slots, H, 64, 512))).astype(np.float32)
    q = rng.standard_normal((ntok, H, 64)); q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((ntok, H, 64)); k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((ntok, H, 64))
    beta = 1 / (1 + np.exp(-rng.standard_normal((ntok, H))))
    decay = 1 / (1 + np.exp(-(rng.standard_normal((ntok, H)) + 3)))
    f = lambda a: a.astype(np.float32)
    return S, f(q), f(k), f(v), f(beta), f(decay)


@pytest.mark.parametrize("readout", ["pre", "post"])
@pytest.mark.parametrize("gated", [False, True])
def test_decode_vs_oracle(kdn, consts, readout, gated):
    S, q, k, v, beta, decay = _decode_inputs(50, 5, 4, 8)
    if not gated:
        decay = None
    slots = np.array([3, 0, 7, 5, 1], np.int64)
    St = to_dev(S)
    out = torch.empty(5, 4, 64, device=DEV)
    kdn.hybrid_recurrent_forward(to_dev(q), to_dev(k), to_dev(v), to_dev(beta), to_dev(decay), St,
                                 to_dev(slots, torch.int64), out, readout=readout)
    step = oracle.decode_step if readout == "pre" else oracle.decode_step_post
    y_ref, S_new = step(S[slots], q, k, v, beta, decay, consts)
    S_ref = S.astype(np.float64).copy()
    S_ref[slots] = S_new
    assert rel_err(out.cpu().numpy(), y_ref) < F32_TOL
    assert fro_rel(St.cpu().numpy(), S_ref) < F32_TOL
    # untouched slots stay bit-identical
    for s in set(range(8)) - set(slots.tolist()):
        assert np.array_equal(St[s].cpu().numpy(), S[s])


def test_decode_matches_reference_post_golden(kdn, proj, golden_dir):
    g = np.load(os.path.join(golden_dir, "decode_post_step.npz"))
    B, H = g["q"].shape[:2]
    St = to_dev(g["S_prev"])
    out = torch.empty(B, H, 64, device=DEV)
    kdn.hybrid_recurrent_forward(to_dev(g["q"]), to_dev(g["k"]), to_dev(g["v"]), to_dev(g["beta"]),
                                 to_dev(g["decay"]), St, torch.arange(B, device=DEV), out, fwht_proj=proj,
                                 readout="post")
    assert rel_err(out.cpu().numpy(), g["y"]) < F32_TOL
    assert fro_rel(St.cpu().numpy(), g["S"]) < F32_TOL


def test_decode_trajectory_matches_prefill(kdn, proj):
    N, T = 3, 40
    q, k, v, beta, decay, S0 = make_inputs(60, N, T, 64, True, True)
    Yp, Sp = kdn.fused_chunked_deltanet_forward(to_dev(q), to_dev(k), to_dev(v), to_dev(beta), to_dev(decay), proj,
                                                64, to_dev(S0), mode="fp32")
    St = to_dev(S0).view(N, 1, 64, 512).clone()
    out = torch.empty(N, 1, 64, device=DEV)
    ys = []
    slots = torch.arange(N, device=DEV, dtype=torch.int32)
    for t in range(T):
        kdn.hybrid_recurrent_forward(to_dev(q[:, t:t + 1]).view(N, 1, 64), to_dev(k[:, t:t + 1]).view(N, 1, 64),
                                     to_dev(v[:, t:t + 1]).view(N, 1, 64), to_dev(beta[:, t:t + 1]),
                                     to_dev(decay[:, t:t + 1]), St, slots, out, fwht_proj=proj)
        ys.append(out[:, 0].clone())
    Yd = torch.stack(ys, 1)
    assert rel_err(Yd.cpu().numpy(), Yp.cpu().numpy()) < 1e-4
    assert fro_rel(St.view(N, 64, 512).cpu().numpy(), Sp.cpu().numpy()) < 1e-4


def test_decode_bf16_state_and_inputs(kdn, consts):
    S, q, k, v, beta, decay = _decode_inputs(70, 6, 2, 6)
    slots = np.arange(6)
    Sb = to_dev(S, torch.bfloat16)
    S_in = Sb.float().cpu().numpy()  # the kernel updates Sb in place
    out = torch.empty(6, 2, 64, device=DEV, dtype=torch.bfloat16)
    kdn.hybrid_recurrent_forward(to_dev(q, torch.bfloat16), to_dev(k, torch.bfloat16), to_dev(v, torch.bfloat16),
                                 to_dev(beta, torch.bfloat16), to_dev(decay, torch.bfloat16), Sb,
                                 to_dev(slots, torch.int64), out)
    y_ref, S_ref = oracle.decode_step(S_in, bf16_round(q), bf16_round(k), bf16_round(v),
                                      bf16_round(beta), bf16_round(decay), consts)
    assert rel_err(out.float().cpu().numpy(), y_ref) < BF16_Y_TOL
    assert fro_rel(Sb.float().cpu().numpy(), S_ref) < BF16_S_TOL


def test_decode_padding_and_out_of_range_slots(kdn):
    from kdn_b200.serving import device_error

    S, q, k, v, beta, _ = _decode_inputs(80, 4, 2, 3)
    St = to_dev(S)
    before = St.clone()
    out = torch.full((4, 2, 64), 7.0, device=DEV)
    slots = torch.tensor([-1, 1, 99, -1], device=DEV, dtype=torch.int64)
    assert device_error() == 0
    kdn.hybrid_recurrent_forward(to_dev(q), to_dev(k), to_dev(v), to_dev(beta), None, St, slots, out)
    assert device_error() != 0  # slot 99 >= 3 recorded, nothing written for it
    assert device_error() == 0  # cleared by the read
    o = out.cpu()
    assert torch.all(o[0] == 0) and torch.all(o[2] == 0) and torch.all(o[3] == 0)
    assert torch.equal(St[0], before[0]) and torch.equal(St[2], before[2])
    assert not torch.equal(St[1], before[1])


def test_fork_state(kdn):
    St = torch.randn(4, 2, 64, 512, device=DEV)
    kdn.fork_recurrent_state(St, 1, 3)
    torch.cuda.synchronize()
    assert torch.equal(St[3], St[1])
    with pytest.raises(RuntimeError, match="out of range"):
        kdn.fork_recurrent_state(St, 0, 4)


# ------------------------------------------------- tensor-core (bf16) path
TC_CASES = [
    # (seed, N, T, gated, init)
    (100, 1, 1, False, False),
    (101, 2, 63, True, True),
    (102, 3, 64, False, True),
    (103, 2, 65, True, False),
    (104, 5, 130, False, False),
    (105, 2, 1000, True, True),
]


@pytest.fixture(params=["fused", "split", "split3"])
def tc_path(request, monkeypatch):
    """Run a tensor-core test on the fused kernel, on the two-phase kernels in one persistent
    launch, and on the two-phase kernels as three separate launches."""
    monkeypatch.setenv("KDN_PREFILL_PATH", "fused" if request.param == "fused" else "split")
    monkeypatch.setenv("KDN_SPLIT_PERSISTENT", "0" if request.param == "split3" else "1")
    return request.param


def split_ws(n, t, rec=238592):
    """Workspace bytes of the two-phase path: chunk records, hand-over flags, abort word."""
    chunks = n * ((t + 63) // 64)
    return chunks * rec + (((chunks + 2 * n) * 4 + 4 + 255) & ~255)


def test_tc_path_selected(kdn, proj, monkeypatch):
    lib = kdn.load()
    s, _ = proj.kdn_projection(DEV)
    assert lib.kdn_chunked_prefill_workspace_size(16, 65536, 64, 64, s, 1) == split_ws(16, 65536)  # few: split
    assert lib.kdn_chunked_prefill_workspace_size(512, 16384, 64, 64, s, 1) == 0  # many sequences: fused
    assert lib.kdn_chunked_prefill_workspace_size(16, 65536, 64, 64, s, 0) > 0   # CUDA-core path
    monkeypatch.setenv("KDN_PREFILL_PATH", "fused")
    assert lib.kdn_chunked_prefill_workspace_size(16, 65536, 64, 64, s, 1) == 0
    monkeypatch.setenv("KDN_PREFILL_PATH", "split")
    assert lib.kdn_chunked_prefill_workspace_size(512, 100, 64, 64, s, 1) == split_ws(512, 100)


@pytest.mark.parametrize("case", TC_CASES)
def test_tc_prefill_vs_oracle(kdn, proj, consts, case, tc_path):
    seed, N, T, gated, init = case
    q, k, v, beta, decay, S0 = make_inputs(seed, N, T, 64, gated, init)
    qb, kb, vb = (to_dev(a, torch.bfloat16) for a in (q, k, v))
    Y, S = kdn.fused_chunked_deltanet_forward(qb, kb, vb, to_dev(beta), to_dev(decay), proj, 64, to_dev(S0),
                                              mode="bf16")
    Yr, Sr = oracle.chunked_deltanet_forward(bf16_round(q), bf16_round(k), bf16_round(v), beta, decay, consts, 64,
                                             S0)
    assert rel_err(Y.float().cpu().numpy(), Yr) < BF16_Y_TOL
    assert fro_rel(S.cpu().numpy(), Sr) < BF16_S_TOL


def test_tc_prefill_fp32_inputs_bf16_mode(kdn, proj, consts, tc_path):
    q, k, v, beta, decay, S0 = make_inputs(110, 2, 200, 64, True, True)
    Y, S = kdn.fused_chunked_deltanet_forward(to_dev(q), to_dev(k), to_dev(v), to_dev(beta), to_dev(decay), proj, 64,
                                              to_dev(S0), mode="bf16")
    assert Y.dtype == torch.float32
    Yr, Sr = oracle.chunked_deltanet_forward(bf16_round(q), bf16_round(k), v, beta, decay, consts, 64, S0)
    assert rel_err(Y.cpu().numpy(), Yr) < BF16_Y_TOL
    assert fro_rel(S.cpu().numpy(), Sr) < BF16_S_TOL


def test_tc_prefill_long_sequence_vs_oracle(kdn, proj, consts, tc_path):
    q, k, v, beta, _, _ = make_inputs(111, 2, 8192, 64, False, False)
    qb, kb, vb = (to_dev(a, torch.bfloat16) for a in (q, k, v))
    Y, S = kdn.fused_chunked_deltanet_forward(qb, kb, vb, to_dev(beta), None, proj, 64, mode="bf16")
    Yr, Sr = oracle.chunked_deltanet_forward(bf16_round(q), bf16_round(k), bf16_round(v), beta, None, consts, 64,
                                             dtype=np.float32)
    assert rel_err(Y.float().cpu().numpy(), Yr) < BF16_Y_TOL
    assert fro_rel(S.cpu().numpy(), Sr) < BF16_S_TOL


@pytest.mark.parametrize("cut", [128, 192])
def test_tc_resume_is_bit_exact(kdn, proj, tc_path, cut):
    """Prefill in two calls, the state carried in fp32, equals one call bit for bit (any chunk-aligned cut)."""
    q, k, v, beta, decay, _ = make_inputs(112, 3, 512, 64, True, False)
    dq, dk, dvv = (to_dev(a, torch.bfloat16) for a in (q, k, v))
    db, dd = to_dev(beta), to_dev(decay)
    Y, S = kdn.fused_chunked_deltanet_forward(dq, dk, dvv, db, dd, proj, 64, mode="bf16")
    Y1, S1 = kdn.fused_chunked_deltanet_forward(dq[:, :cut], dk[:, :cut], dvv[:, :cut], db[:, :cut], dd[:, :cut],
                                                proj, 64, mode="bf16")
    Y2, S2 = kdn.fused_chunked_deltanet_forward(dq[:, cut:], dk[:, cut:], dvv[:, cut:], db[:, cut:], dd[:, cut:],
                                                proj, 64, S1, mode="bf16")
    assert torch.equal(torch.cat([Y1, Y2], 1), Y)
    assert torch.equal(S2, S)


def test_tc_full_config1_vs_fp32_path(kdn, proj, tc_path):
    """Config 1 at full size (16 heads x 65536 tokens): the tensor-core path
    against the exact fp32 CUDA-core path (itself pinned to the oracle above)."""
    H, T = 16, 65536
    g = torch.Generator(device=DEV).manual_seed(7)
    q = torch.nn.functional.normalize(torch.randn(H, T, 64, generator=g, device=DEV), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(H, T, 64, generator=g, device=DEV), dim=-1).bfloat16()
    v = torch.randn(H, T, 64, generator=g, device=DEV).bfloat16()
    beta = torch.sigmoid(torch.randn(H, T, generator=g, device=DEV))
    Yt, St = kdn.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, 64, mode="bf16")
    Yf, Sf = kdn.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, 64, mode="fp32")
    ey = ((Yt.float() - Yf.float()).norm(dim=-1) / Yf.float().norm(dim=-1).clamp_min(1e-30)).max().item()
    es = ((St - Sf).norm() / Sf.norm()).item()
    assert ey < BF16_Y_TOL, ey
    assert es < BF16_S_TOL, es


def test_tc_fused_and_split_paths_agree(kdn, proj, monkeypatch):
    """The two tensor-core schedules compute the same chunk algebra; they differ
    only in where (I + A)^-1 is applied, i.e. in fp16 rounding."""
    q, k, v, beta, decay, S0 = make_inputs(120, 3, 700, 64, True, True)
    args = [to_dev(a, torch.bfloat16) for a in (q, k, v)] + [to_dev(beta), to_dev(decay), proj, 64, to_dev(S0)]
    out = {}
    for path, persistent in (("fused", "1"), ("split", "1"), ("split", "0")):
        monkeypatch.setenv("KDN_PREFILL_PATH", path)
        monkeypatch.setenv("KDN_SPLIT_PERSISTENT", persistent)
        out[path + persistent] = kdn.fused_chunked_deltanet_forward(*args, mode="bf16")
    (Yf, Sf), (Ys, Ss), (Y3, S3) = out["fused1"], out["split1"], out["split0"]
    assert rel_err(Ys.float().cpu().numpy(), Yf.float().cpu().numpy()) < BF16_Y_TOL
    assert fro_rel(Ss.cpu().numpy(), Sf.cpu().numpy()) < BF16_S_TOL
    assert torch.equal(Ys, Y3) and torch.equal(Ss, S3)  # same arithmetic, one launch or three
    from kdn_b200.serving import device_error

    assert device_error() == 0


# ------------------------------------------------------------------ host streaming
@pytest.mark.parametrize("mode,seg", [("bf16", 256), ("fp32", 192)])
def test_streamed_host_prefill_equals_one_call(kdn, proj, mode, seg):
    """Host tensors streamed through the GPU in segments give what one device call gives
    (the state is carried between segments in fp32; ragged last segment)."""
    dt = torch.bfloat16 if mode == "bf16" else torch.float32
    q, k, v, beta, decay, S0 = make_inputs(31, 3, 1000, gated=True, init=True)
    h = lambda a, d=torch.float32: torch.from_numpy(a).to(d).pin_memory()
    yh, Sh = kdn.fused_chunked_deltanet_forward(h(q, dt), h(k, dt), h(v, dt), h(beta), h(decay), proj, 64, h(S0),
                                                mode=mode, device=DEV, segment_tokens=seg)
    assert not yh.is_cuda and not Sh.is_cuda
    yd, Sd = kdn.fused_chunked_deltanet_forward(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), to_dev(beta),
                                                to_dev(decay), proj, 64, to_dev(S0), mode=mode)
    torch.cuda.synchronize()
    # same chunks, same arithmetic: identical up to the path's own run-to-run determinism
    assert rel_err(yh.float().numpy(), yd.float().cpu().numpy()) < (1e-3 if mode == "bf16" else 1e-6)
    assert fro_rel(Sh.numpy(), Sd.cpu().numpy()) < (1e-3 if mode == "bf16" else 1e-6)


def test_host_tensors_need_a_device(kdn, proj):
    x = torch.zeros(1, 8, 64)
    with pytest.raises(RuntimeError, match="device="):
        kdn.fused_chunked_deltanet_forward(x, x, x, torch.zeros(1, 8), None, proj)
