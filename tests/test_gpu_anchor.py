"""The softmax anchors' prefill kernels (kdn_anchor_qkv, kdn_varlen_causal_attention).

CPU: argument checks of the C entries (no device work).
GPU:
  * anchor_qkv against the layer's torch restatement of rotate-half rotary (the fp32 verification
    path, layers/hybrid_kernel_deltanet_block.py ``rotary``): q head-major and token-major, k and v in
    the cache rows, positions offset by start_pos; every element within one bf16 rounding;
  * varlen causal attention of packed sequences (lengths on both sides of the 128-key tile and
    256-query block edges, permuted cache rows, cache positions past each length filled with large
    values that the causal mask must hide) against float64 softmax attention of the same bf16 inputs,
    at two score scales (the larger one moves the row maximum across key tiles): max error <= 1e-2 of
    the largest output, mean error <= 1e-3 of it;
  * the LM anchor layer's bf16 prefill on the libkdn path equals its fp32 torch path within bf16
    rounding of the output projection.
"""

import math

import pytest
import torch


def test_anchor_argument_checks(lib):
    P = 4096
    assert lib.kdn_anchor_qkv(P, 1, P, None, None, 2, 10, 4, 32, 1e4, P, 1, P, P, 2, 64, None) == 2  # d_head
    assert lib.kdn_anchor_qkv(P, 0, P, None, None, 2, 10, 4, 64, 1e4, P, 1, P, P, 2, 64, None) == 2  # fp32
    assert lib.kdn_anchor_qkv(P, 1, None, None, None, 2, 10, 4, 64, 1e4, P, 1, P, P, 2, 64, None) == 1
    assert lib.kdn_anchor_qkv(P, 1, P, None, None, 2, 10, 4, 64, -1.0, P, 1, P, P, 2, 64, None) == 1  # theta
    assert lib.kdn_anchor_qkv(P, 1, P, None, None, 2, 0, 4, 64, 1e4, P, 1, P, P, 2, 64, None) == 0   # no tokens
    a = lambda **k: lib.kdn_varlen_causal_attention(
        k.get("q", P), P, P, k.get("dt", 1), P, None, 2, k.get("n", 10), 4, k.get("dh", 64), 2, k.get("L", 64),
        k.get("ms", 8), k.get("o", P), None)
    assert a(dh=32) == 2
    assert a(dt=0) == 2
    assert a(ms=65) == 1            # max_seqlen past the cache
    assert a(q=P + 8) == 1          # misaligned
    assert a(o=None) == 1
    assert a(L=1 << 28) == 2        # cache rows past 32-bit tensor-map coordinates
    assert a(n=0) == 0


def _rotary_ref(x, pos, theta):
    from kdn_b200.layers.hybrid_kernel_deltanet_block import rotary

    return rotary(x, pos, theta)


@pytest.mark.gpu
def test_anchor_qkv_matches_torch_rotary():
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(11)
    H, L, theta = 3, 300, 10000.0
    lens = [5, 130, 1, 77]
    starts = [0, 17, 200, 3]
    rows = [2, 0, 3, 1]
    n = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), device="cuda", dtype=torch.int64)
    qkv = torch.randn(n, 3 * H * 64, generator=g, device="cuda").to(torch.bfloat16)
    kc = torch.zeros(4, H, L, 64, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    st = torch.tensor(starts, device="cuda")
    rw = torch.tensor(rows, device="cuda")
    q_hm = glue.anchor_qkv(qkv, cu, H, theta, kc, vc, rw, st, q_head_major=True)
    q_tm = glue.anchor_qkv(qkv, cu, H, theta, kc, vc, rw, st, q_head_major=False)
    assert torch.equal(q_hm.transpose(0, 1), q_tm)
    pos = torch.cat([torch.arange(n_, device="cuda") + s for n_, s in zip(lens, starts)])
    q, k, v = qkv.view(n, 3, H, 64).unbind(1)
    rq, rk = _rotary_ref(q, pos, theta), _rotary_ref(k, pos, theta)
    tol = lambda ref: 2.0 ** -8 * ref.float().abs() + 1e-6
    assert bool(((q_tm.float() - rq.float()).abs() <= tol(rq)).all())
    c = 0
    for i, n_ in enumerate(lens):
        seg = slice(c, c + n_)
        ck = kc[rows[i], :, starts[i]:starts[i] + n_].transpose(0, 1)
        cv = vc[rows[i], :, starts[i]:starts[i] + n_].transpose(0, 1)
        assert bool(((ck.float() - rk[seg].float()).abs() <= tol(rk[seg])).all())
        assert torch.equal(cv, v[seg])
        c += n_


def _attention_ref(q, k, v):
    """float64 causal softmax attention, q/k/v [T, H, 64] -> [T, H, 64]."""
    T = q.shape[0]
    qd, kd, vd = (t.double().transpose(0, 1) for t in (q, k, v))  # [H, T, 64]
    s = qd @ kd.transpose(1, 2) / 8.0
    mask = torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1)
    s.masked_fill_(mask, float("-inf"))
    return (torch.softmax(s, dim=-1) @ vd).transpose(0, 1)


@pytest.mark.gpu
@pytest.mark.parametrize("scale", [1.0, 4.0])
def test_varlen_causal_attention_vs_float64(scale):
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(int(scale * 10))
    H = 2
    lens = [1, 127, 128, 129, 255, 256, 257, 700, 1500]
    rows = [4, 0, 8, 2, 6, 1, 3, 7, 5]
    L = 1600
    n = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), device="cuda", dtype=torch.int64)
    q = (torch.randn(H, n, 64, generator=g, device="cuda") * scale).to(torch.bfloat16)
    # cache positions past every length hold large values: a key the mask fails to hide shows up
    kc = (torch.randn(9, H, L, 64, generator=g, device="cuda") * 30).to(torch.bfloat16)
    vc = (torch.randn(9, H, L, 64, generator=g, device="cuda") * 30).to(torch.bfloat16)
    ks, vs = [], []
    for i, n_ in enumerate(lens):
        k_i = torch.randn(n_, H, 64, generator=g, device="cuda").to(torch.bfloat16)
        v_i = torch.randn(n_, H, 64, generator=g, device="cuda").to(torch.bfloat16)
        kc[rows[i], :, :n_] = k_i.transpose(0, 1)
        vc[rows[i], :, :n_] = v_i.transpose(0, 1)
        ks.append(k_i)
        vs.append(v_i)
    out = glue.varlen_causal_attention(q, kc, vc, cu, max(lens), torch.tensor(rows, device="cuda"))
    assert out.shape == (n, H, 64) and bool(torch.isfinite(out.float()).all())
    c = 0
    for i, n_ in enumerate(lens):
        ref = _attention_ref(q[:, c:c + n_].transpose(0, 1), ks[i], vs[i])
        err = (out[c:c + n_].double() - ref).abs()
        big = float(ref.abs().max())
        assert float(err.max()) <= 1e-2 * big, (n_, float(err.max()), big)
        assert float(err.mean()) <= 1e-3 * big, (n_, float(err.mean()), big)
        c += n_


@pytest.mark.gpu
def test_anchor_layer_bf16_path_matches_fp32_path():
    """SoftmaxAnchor.prefill: bf16 weights on libkdn (projection, rotary, varlen attention) against the
    fp32 verification path (torch rotary + SDPA) on the same bf16-rounded weights and inputs."""
    from kdn_b200.layers.hybrid_kernel_deltanet_block import SoftmaxAnchor

    torch.manual_seed(3)
    d, H = 256, 4
    lay = SoftmaxAnchor(d, H).cuda()
    with torch.no_grad():
        for p in lay.parameters():
            p.copy_(torch.randn_like(p) / math.sqrt(p.shape[1]))
    lens = [100, 300, 7]
    cu = [0, 100, 400, 407]
    x = torch.randn(cu[-1], d, device="cuda").to(torch.bfloat16)
    lb = SoftmaxAnchor(d, H).cuda().to(torch.bfloat16)
    lb.load_state_dict({k: v.to(torch.bfloat16) for k, v in lay.state_dict().items()})
    lf = SoftmaxAnchor(d, H).cuda()
    lf.load_state_dict({k: v.to(torch.bfloat16).float() for k, v in lay.state_dict().items()})
    kb = torch.zeros(3, H, 512, 64, device="cuda", dtype=torch.bfloat16)
    kf = torch.zeros(3, H, 512, 64, device="cuda")
    yb = lb.prefill(x, cu, kb, torch.zeros_like(kb), [0, 1, 2])
    yf = lf.prefill(x.float(), cu, kf, torch.zeros_like(kf), [0, 1, 2])
    err = float((yb.float() - yf).abs().max())
    assert err <= 3e-2 * float(yf.abs().max()), err
    assert float((kb.float() - kf).abs().max()) <= 2e-2 * float(kf.abs().max())
