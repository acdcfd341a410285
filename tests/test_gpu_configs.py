"""Parity at the benchmark configurations' own sizes (configs 0-3 of the build's baseline).

Each test runs libkdn on the GPU through the production path the library picks for that shape
and compares with the CPU oracle (oracle/chunked.py, oracle/recurrence.py, pinned to the
reference's golden vectors) on the same seeded inputs:

  config 0  B=1, H=4, T=2048, fp32 mode             all heads vs the float64 oracle, <= 1e-4
  config 1  B=1, H=16, T=65536, bf16 inputs         two heads of the full 16-head call vs the oracle
                                                    (float32, on the bf16-rounded inputs):
                                                    outputs <= 2e-2, state <= 1e-2
  config 2  B=32, H=16, T=16384 (512 scans)         the many-sequence kernel (chosen at N >= SMs)
                                                    on 160 scans x 2048 tokens vs the oracle, and
                                                    two scans of the full 512 x 16384 call vs the
                                                    oracle plus the whole call vs the fp32 path
  config 3  64 streams x 16 heads, fp32 state       three decode steps on all 1024 heads vs the
                                                    float64 decode step, and the 1024-step
                                                    trajectory vs the fp32 prefill of the same tokens

Inputs follow the configurations: q, k ~ N(0, 1) then L2-normalised per head vector, v ~ N(0, 1),
beta = sigmoid(N(0, 1)), no decay, zero initial state (config 3: state ~ N(0, 0.02^2)).
Set KDN_PARITY_LOG=<file> to append each measured error as a JSON line.
"""

import json
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


def errors(Y, Yref):
    """Error figures of outputs Y against Yref ([N, T, d] float arrays or tensors, rows = last axis):
      fro     max over sequences of ||Y_n - Yref_n||_F / ||Yref_n||_F -- the reference's own output
              metric (tests/test_fused_kernel.py:93-95 takes the Frobenius ratio over the tensor)
      row     max over rows of ||y - y_ref|| / ||y_ref||, every row
      row_wc  the same over rows whose reference norm is at least 0.1 x the RMS row norm of their
              sequence: a relative error of a near-zero row measures fp16 rounding of the features,
              not the algorithm (its absolute error is as small as every other row's)
    plus the worst row's norm relative to its sequence's RMS row norm."""
    Y = torch.as_tensor(Y).double()
    R = torch.as_tensor(Yref).double()
    d = (Y - R).norm(dim=-1)
    n = R.norm(dim=-1)
    rms = n.pow(2).mean(dim=-1, keepdim=True).sqrt()
    rel = d / n.clamp_min(1e-30)
    wc = n >= 0.1 * rms
    worst = int(rel.argmax())
    fro = ((Y - R).flatten(1).norm(dim=-1) / R.flatten(1).norm(dim=-1).clamp_min(1e-30)).max()
    return {"fro": float(fro), "row": float(rel.max()), "row_wc": float(rel[wc].max()),
            "worst_row_norm_over_rms": float((n / rms).flatten()[worst])}


def log(case, **errs):
    path = os.environ.get("KDN_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": case, **errs}) + "\n")


def device_inputs(seed, N, T, dtype):
    """Seeded config inputs generated on the GPU: q, k, v [N, T, 64] in `dtype`, beta [N, T] fp32."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(N, T, 64, generator=g, device=DEV), dim=-1).to(dtype)
    k = torch.nn.functional.normalize(torch.randn(N, T, 64, generator=g, device=DEV), dim=-1).to(dtype)
    v = torch.randn(N, T, 64, generator=g, device=DEV).to(dtype)
    beta = torch.sigmoid(torch.randn(N, T, generator=g, device=DEV))
    return q, k, v, beta


def host(t, rows=None):
    t = t if rows is None else t[rows]
    return t.float().cpu().numpy()


def prefill_path(kdn, proj, N, T):
    """'split' / 'fused' / 'simt': which bf16 kernel family the library runs for [N, T]."""
    lib = kdn.load()
    s, _ = proj.kdn_projection(DEV)
    return "split" if lib.kdn_chunked_prefill_workspace_size(N, T, 64, 64, s, 1) > 0 else "fused"


def test_config0_fp32_full(kdn, proj, consts):
    q, k, v, beta = device_inputs(0, 4, 2048, torch.float32)
    Y, S = kdn.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, 64, mode="fp32")
    Yr, Sr = oracle.chunked_deltanet_forward(host(q), host(k), host(v), host(beta), None, consts, 64)
    ey, es = rel_err(host(Y), Yr), fro_rel(host(S), Sr)
    log("config0 fp32 B=1 H=4 T=2048", y=ey, S=es)
    assert ey < F32_TOL, ey
    assert es < F32_TOL, es


def test_config1_bf16_two_heads_vs_oracle(kdn, proj, consts):
    N, T = 16, 65536
    assert prefill_path(kdn, proj, N, T) == "split"
    q, k, v, beta = device_inputs(1, N, T, torch.bfloat16)
    Y, S = kdn.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, 64, mode="bf16")
    heads = [0, 9]
    Yr, Sr = oracle.chunked_deltanet_forward(host(q, heads), host(k, heads), host(v, heads), host(beta, heads), None,
                                             consts, 64, dtype=np.float32)
    ey, es = rel_err(host(Y, heads), Yr), fro_rel(host(S, heads), Sr)
    # growth with length: the same two heads over the first 8192 tokens only
    ey8 = rel_err(host(Y, heads)[:, :8192], Yr[:, :8192])
    log("config1 bf16 H=16 T=65536 (heads 0, 9 vs oracle)", y=ey, S=es, y_first_8192=ey8)
    assert ey < BF16_Y_TOL, ey
    assert es < BF16_S_TOL, es


def test_config2_many_sequence_kernel_vs_oracle(kdn, proj, consts):
    N, T = 160, 2048
    assert prefill_path(kdn, proj, N, T) == "fused"
    q, k, v, beta = device_inputs(2, N, T, torch.bfloat16)
    Y, S = kdn.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, 64, mode="bf16")
    Yr, Sr = oracle.chunked_deltanet_forward(host(q), host(k), host(v), host(beta), None, consts, 64,
                                             dtype=np.float32)
    ey, es = rel_err(host(Y), Yr), fro_rel(host(S), Sr)
    log("config2 kernel bf16 N=160 T=2048 vs oracle", y=ey, S=es, **errors(host(Y), Yr))
    assert ey < BF16_Y_TOL, ey
    assert es < BF16_S_TOL, es


def test_config2_full_size(kdn, proj, consts):
    N, T = 512, 16384
    assert prefill_path(kdn, proj, N, T) == "fused"
    q, k, v, beta = device_inputs(3, N, T, torch.bfloat16)
    Yt, St = kdn.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, 64, mode="bf16")
    rows = [5, 300]
    Yr, Sr = oracle.chunked_deltanet_forward(host(q, rows), host(k, rows), host(v, rows), host(beta, rows), None,
                                             consts, 64, dtype=np.float32)
    ey, es = rel_err(host(Yt, rows), Yr), fro_rel(host(St, rows), Sr)
    Yf, Sf = kdn.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, 64, mode="fp32")
    e_all = errors(Yt.float(), Yf.float())
    es_all = ((St - Sf).flatten(1).norm(dim=-1) / Sf.flatten(1).norm(dim=-1)).max().item()
    log("config2 bf16 N=512 T=16384", y_rows_vs_oracle=ey, S_rows_vs_oracle=es,
        **{f"y_all_vs_fp32_{k}": v for k, v in e_all.items()}, S_all_vs_fp32=es_all)
    assert ey < BF16_Y_TOL, ey
    assert es < BF16_S_TOL, es
    assert e_all["fro"] < BF16_Y_TOL, e_all
    assert e_all["row_wc"] < BF16_Y_TOL, e_all
    assert es_all < BF16_S_TOL, es_all


def test_config2_eight_gpu_shard(kdn, proj, consts):
    """The per-GPU shard of config 2 at 8 GPUs (64 scans x 16384): the two-phase path."""
    N, T = 64, 16384
    assert prefill_path(kdn, proj, N, T) == "split"
    q, k, v, beta = device_inputs(6, N, T, torch.bfloat16)
    Yt, St = kdn.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, 64, mode="bf16")
    rows = [0, 63]
    Yr, Sr = oracle.chunked_deltanet_forward(host(q, rows), host(k, rows), host(v, rows), host(beta, rows), None,
                                             consts, 64, dtype=np.float32)
    e_or = errors(host(Yt, rows), Yr)
    es = fro_rel(host(St, rows), Sr)
    Yf, Sf = kdn.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, 64, mode="fp32")
    e_all = errors(Yt.float(), Yf.float())
    log("config2 shard bf16 N=64 T=16384", **{f"y_rows_vs_oracle_{k}": v for k, v in e_or.items()},
        S_rows_vs_oracle=es, **{f"y_all_vs_fp32_{k}": v for k, v in e_all.items()})
    assert e_or["row"] < BF16_Y_TOL, e_or
    assert es < BF16_S_TOL, es
    assert e_all["fro"] < BF16_Y_TOL and e_all["row_wc"] < BF16_Y_TOL, e_all


def _decode_setup(seed, streams=64, heads=16, steps=3):
    g = torch.Generator(device=DEV).manual_seed(seed)
    S0 = 0.02 * torch.randn(streams, heads, 64, 512, generator=g, device=DEV)
    q = torch.nn.functional.normalize(torch.randn(steps, streams, heads, 64, generator=g, device=DEV), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(steps, streams, heads, 64, generator=g, device=DEV), dim=-1)
    v = torch.randn(steps, streams, heads, 64, generator=g, device=DEV)
    beta = torch.sigmoid(torch.randn(steps, streams, heads, generator=g, device=DEV))
    return S0, q, k, v, beta


def test_config3_decode_all_heads_vs_oracle(kdn, proj, consts):
    S0, q, k, v, beta = _decode_setup(4, steps=3)
    states = S0.clone()
    out = torch.empty(64, 16, 64, device=DEV)
    slots = torch.arange(64, device=DEV)
    S_ref = S0.double().cpu().numpy()
    worst_y = 0.0
    for t in range(3):
        kdn.hybrid_recurrent_forward(q[t], k[t], v[t], beta[t], None, states, slots, out, fwht_proj=proj)
        y_ref, S_ref = oracle.decode_step(S_ref, host(q[t]), host(k[t]), host(v[t]), host(beta[t]), None, consts)
        worst_y = max(worst_y, rel_err(host(out), y_ref))
    es = fro_rel(host(states), S_ref)
    log("config3 decode 64x16, 3 steps vs oracle", y=worst_y, S=es)
    assert worst_y < F32_TOL, worst_y
    assert es < F32_TOL, es


def test_config3_trajectory_vs_prefill(kdn, proj):
    """1024 decode steps on all 64 x 16 heads equal the fp32 prefill of the same 1024 tokens
    from the same initial states (readout before the update in both)."""
    steps = 1024
    S0, q, k, v, beta = _decode_setup(5, steps=steps)
    states = S0.clone()
    out = torch.empty(64, 16, 64, device=DEV)
    slots = torch.arange(64, device=DEV)
    ys = torch.empty(steps, 64, 16, 64, device=DEV)
    for t in range(steps):
        kdn.hybrid_recurrent_forward(q[t], k[t], v[t], beta[t], None, states, slots, out, fwht_proj=proj)
        ys[t].copy_(out)
    flat = lambda x: x.permute(1, 2, 0, 3).reshape(64 * 16, steps, -1).contiguous()
    Yp, Sp = kdn.fused_chunked_deltanet_forward(flat(q), flat(k), flat(v), beta.permute(1, 2, 0).reshape(1024, steps),
                                                None, proj, 64, S0.reshape(1024, 64, 512), mode="fp32")
    ey = rel_err(host(flat(ys)), host(Yp))
    es = fro_rel(host(states.reshape(1024, 64, 512)), host(Sp))
    log("config3 decode 64x16, 1024-step trajectory vs fp32 prefill", y=ey, S=es)
    assert ey < F32_TOL, ey
    assert es < F32_TOL, es
