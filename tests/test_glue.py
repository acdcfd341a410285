"""Element-wise kernels of the hybrid block (kdn_rmsnorm, kdn_add_rmsnorm, kdn_swiglu, kdn_mixer_inputs) and
its dense projection (kdn_linear).

CPU: argument checks of the C entries (no device work).  GPU: each kernel against the same
formula in torch fp32 -- fp32 storage within 1e-6 relative, bf16 storage within one bf16
rounding of the fp32 result (2^-8 relative).
"""

import pytest
import torch


def test_glue_argument_checks(lib):
    P = 4096
    assert lib.kdn_rmsnorm(P, 1, P, 0, P, 4, 2052, 1e-6, None) == 2       # d not a multiple of 8 (bf16)
    assert lib.kdn_rmsnorm(P + 4, 1, P, 0, P, 4, 2048, 1e-6, None) == 1   # misaligned x
    assert lib.kdn_rmsnorm(P, 5, P, 0, P, 4, 2048, 1e-6, None) == 1       # bad dtype
    assert lib.kdn_rmsnorm(P, 1, P, 0, P, 0, 2048, 1e-6, None) == 0       # nothing to do
    Q, R, O = P + 65536, P + 2 * 65536, P + 3 * 65536
    assert lib.kdn_add_rmsnorm(P, Q, 1, R, 0, None, O, 4, 2048, 1e-6, None) == 1   # h_out NULL with a residual
    assert lib.kdn_add_rmsnorm(P, Q, 1, R, 0, P, P, 4, 2048, 1e-6, None) == 1      # out aliases x / h_out
    assert lib.kdn_add_rmsnorm(P, Q + 8, 1, R, 0, P, O, 4, 2048, 1e-6, None) == 1  # misaligned residual
    assert lib.kdn_add_rmsnorm(P, Q, 1, R, 0, P, O, 4, 2044, 1e-6, None) == 2      # d not a multiple of 8
    assert lib.kdn_add_rmsnorm(P, Q, 1, R, 0, P, O, 0, 2048, 1e-6, None) == 0      # nothing to do
    assert lib.kdn_swiglu(P, P, 0, 4, 6, None) == 2                        # d_ff not a multiple of 4 (fp32)
    assert lib.kdn_swiglu(None, P, 0, 4, 8, None) == 1
    assert lib.kdn_mixer_inputs(P, 1, 4, 2, 32, 0, P, 0, None, 0, P, P, P, P, P, None) == 2   # d_head must be 64
    assert lib.kdn_mixer_inputs(P, 1, 4, 2, 64, 0, None, 0, None, 0, P, P, P, P, P, None) == 1
    assert lib.kdn_mixer_inputs(P, 1, 4, 2, 64, 385, P, 0, None, 0, P, P, P, P, P, None) == 1  # z_ld below the row (386)
    assert lib.kdn_mixer_inputs(P, 1, 0, 2, 64, 0, P, 0, None, 0, P, P, P, P, P, None) == 0
    assert lib.kdn_linear(P, P, P, 1, 4, 100, 96, 0, None) == 2      # K not a multiple of 64
    assert lib.kdn_linear(P, P, P, 1, 4, 100, 128, 99, None) == 1    # ldo below N
    assert lib.kdn_linear(P, P, P, 1, 4, 100, 128, 100, None) == 1   # ldo not a multiple of 16 bytes (bf16)
    assert lib.kdn_linear(P, P, P, 0, 4, 100, 128, 102, None) == 1   # ... nor (fp32)
    assert lib.kdn_linear(P + 2, P, P, 1, 4, 100, 128, 0, None) == 1  # misaligned x
    assert lib.kdn_linear(P, P, None, 1, 4, 96, 128, 0, None) == 1   # no output
    assert lib.kdn_linear(P, P, P, 5, 4, 96, 128, 0, None) == 1      # bad dtype
    assert lib.kdn_linear(P, P, P, 1, 0, 96, 128, 0, None) == 0      # nothing to do
    assert lib.kdn_linear_swiglu(P, P, P, 4, 192, 128, 0, None) == 2   # d_ff not a multiple of 128
    assert lib.kdn_linear_swiglu(P, P, P, 4, 256, 96, 0, None) == 2    # K not a multiple of 64
    assert lib.kdn_linear_swiglu(P, P, None, 4, 256, 128, 0, None) == 1
    assert lib.kdn_linear_swiglu(P, P, P, 4, 256, 128, 255, None) == 1  # ldo below d_ff
    assert lib.kdn_linear_swiglu(P, P, P, 0, 256, 128, 0, None) == 0
    assert lib.kdn_decode_attention(P, P, P, P, P, 1, 2, 4, 100, 32, P, 1 << 20, None) == 2   # d_head 64 only
    assert lib.kdn_decode_attention(P, None, P, P, P, 1, 2, 4, 100, 64, P, 1 << 20, None) == 1
    assert lib.kdn_decode_attention(P, P, P, P, P, 1, 2, 4, 100, 64, P, 8, None) == 4        # workspace too small
    assert lib.kdn_decode_attention(P, P, P, P, P, 1, 0, 4, 100, 64, None, 0, None) == 0     # no sequences
    assert lib.kdn_decode_attention_workspace_size(2, 4, 2000) == 4 * 2 * 4 * 2 * 66  # 1024 keys per split


def _close(got, ref, dtype):
    tol = 1e-6 if dtype == torch.float32 else 2.0 ** -8
    return bool(((got.float() - ref).abs() <= tol * ref.abs() + 1e-6).all())


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rmsnorm_and_swiglu(dtype):
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(333, 2048, generator=g, device="cuda").to(dtype)
    w = (1 + 0.1 * torch.randn(2048, generator=g, device="cuda")).to(dtype)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert _close(glue.rms_norm(x, w, 1e-6), ref, dtype)
    gu = torch.randn(77, 2 * 8192, generator=g, device="cuda").to(dtype)
    gf = gu.float()
    ref = torch.nn.functional.silu(gf[:, :8192]) * gf[:, 8192:]
    assert _close(glue.swiglu_product(gu), ref, dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 2048, 4104, 8192])
def test_add_rmsnorm(dtype, d):
    """h = x + r rounded to the storage dtype (bit-equal to torch's add), then RMSNorm(h); rows of
    d <= 256 vectors per warp stay in registers, longer ones (4104, 8192; fp32 2048) are read back.
    Weights of another dtype (fp32 weights on bf16 rows) take the element-load path."""
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(19, d, generator=g, device="cuda").to(dtype)
    r = torch.randn(19, d, generator=g, device="cuda").to(dtype)
    for w in ((1 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(dtype),
              1 + 0.1 * torch.randn(d, generator=g, device="cuda")):
        h, out = glue.add_rms_norm(x, r, w, 1e-6)
        href = x + r
        assert torch.equal(h, href)
        hf = href.float()
        ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
        assert _close(out, ref, dtype)
        assert _close(glue.rms_norm(x, w, 1e-6), x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True)
                                                                          + 1e-6) * w.float(), dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,H", [(torch.float32, 3), (torch.bfloat16, 32)])
def test_mixer_inputs(dtype, H):
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(1)
    n = 129
    z = torch.randn(n, 3 * H * 64 + H, generator=g, device="cuda").to(dtype)
    ld = torch.randn(H, generator=g, device="cuda")
    q, k, v, beta, decay = glue.mixer_inputs(z, H, ld)
    zf = z.float()
    rq = torch.nn.functional.normalize(zf[:, :H * 64].view(n, H, 64), dim=-1)
    rk = torch.nn.functional.normalize(zf[:, H * 64:2 * H * 64].view(n, H, 64), dim=-1)
    assert _close(q, rq, dtype) and _close(k, rk, dtype)
    assert torch.equal(v, z[:, 2 * H * 64:3 * H * 64].reshape(n, H, 64))
    assert _close(beta, torch.sigmoid(zf[:, 3 * H * 64:]), torch.float32)
    assert _close(decay, torch.sigmoid(ld).expand(n, H), torch.float32)


@pytest.mark.gpu
def test_mixer_inputs_head_major_layout():
    """With cu_seqlens the split writes the ragged head-major layout: the same values as the packed split
    moved by kdn_ragged_transpose."""
    from kdn_b200.kernels import glue
    from kdn_b200.serving.ragged import _to_head_major
    from kdn_b200 import _lib

    g = torch.Generator(device="cuda").manual_seed(4)
    H, lens = 3, [5, 1, 40, 17]
    n = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), device="cuda", dtype=torch.int64)
    z = torch.randn(n, 3 * H * 64 + H, generator=g, device="cuda").to(torch.bfloat16)
    ld = torch.randn(H, generator=g, device="cuda")
    packed = glue.mixer_inputs(z, H, ld)
    hm = glue.mixer_inputs(z, H, ld, cu_seqlens=cu)
    lib = _lib.load()
    for a, b in zip(packed, hm):
        moved = _to_head_major(lib, a.contiguous(), cu, len(lens), H, torch.device("cuda"))
        assert torch.equal(moved.view(-1), b.reshape(-1))


@pytest.mark.gpu
def test_mixer_inputs_strided_rows():
    """A padded projection output (rows wider than 3 H 64 + H) splits like its contiguous copy."""
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(2)
    n, H = 70, 2
    wide = torch.randn(n, 3 * H * 64 + H + 6, generator=g, device="cuda").to(torch.bfloat16)
    z = wide[:, :3 * H * 64 + H]
    ld = torch.randn(H, generator=g, device="cuda")
    for a, b in zip(glue.mixer_inputs(z, H, ld), glue.mixer_inputs(z.contiguous(), H, ld)):
        assert torch.equal(a, b)


# (M, N, K): decode-size rows (GEMV, 4/8/16-row buckets and a second pass), the GEMM's partial tiles at the
# M and N edges (N below one 256-column tile, odd N, the LM's 6176 / 32000), and K of one and many steps
_LINEAR_SHAPES = [(1, 263, 128), (3, 2048, 2048), (8, 6176, 2048), (13, 386, 128), (16, 2048, 8192), (40, 7, 64),
                  (64, 512, 256), (65, 128, 256), (200, 386, 128), (300, 263, 128), (1000, 6176, 2048),
                  (777, 32000, 2048), (2048, 2048, 8192)]


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", _LINEAR_SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_linear_vs_fp32_matmul(M, N, K, out_dtype):
    """kdn_linear against torch's fp32 product of the same bf16 operands: fp32 output within 1e-5 of the
    largest |x||w| row-column product scale (accumulation order only), bf16 output within one bf16 rounding."""
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") / K ** 0.5).to(torch.bfloat16)
    y = glue.linear(x, w, out_dtype=out_dtype)
    ref = x.double() @ w.double().t()
    assert y.shape == (M, N) and y.dtype == out_dtype
    scale = float((x.double().norm(dim=1).max() * w.double().norm(dim=1).max()))
    err = (y.double() - ref).abs()
    if out_dtype == torch.float32:
        assert float(err.max()) <= 1e-5 * scale
    else:
        assert bool((err <= 2.0 ** -8 * ref.abs() + 1e-5 * scale).all())


@pytest.mark.gpu
@pytest.mark.parametrize("M,F,K", [(65, 128, 64), (300, 384, 256), (1000, 8192, 2048), (129, 256, 8192)])
def test_linear_swiglu_vs_fp32(M, F, K):
    """The fused gate/up GEMM + SwiGLU epilogue against silu(g) * u from the float64 products of the same
    bf16 operands: within one bf16 rounding plus 1e-5 of the output scale."""
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(M + F)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(2 * F, K, generator=g, device="cuda") / K ** 0.5).to(torch.bfloat16)
    y = glue.linear_swiglu(x, glue.swiglu_interleave(w))
    gu = x.double() @ w.double().t()
    ref = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
    assert y.shape == (M, F) and y.dtype == torch.bfloat16
    assert bool(((y.double() - ref).abs() <= 2.0 ** -8 * ref.abs() + 1e-5 * float(ref.abs().max())).all())


@pytest.mark.gpu
def test_linear_batched_input_and_launch_forms():
    """A [B, T, K] input gives the [B, T, N] product; the GEMV (M <= 64) and GEMM forms agree on the
    same rows."""
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(2, 70, 256, generator=g, device="cuda").to(torch.bfloat16)
    w = torch.randn(384, 256, generator=g, device="cuda").to(torch.bfloat16)
    y = glue.linear(x, w, out_dtype=torch.float32)
    assert y.shape == (2, 70, 384)
    rows = glue.linear(x.reshape(140, 256)[:50].contiguous(), w, out_dtype=torch.float32)
    assert float((y.reshape(140, 384)[:50] - rows).abs().max()) <= 1e-5 * float(rows.abs().max())


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_attention(dtype):
    """Split-K one-token attention over ragged cache lengths (split boundaries 1023/1024/1025) against
    a float64 softmax; a length past the cache gives a zero row."""
    from kdn_b200.kernels import glue

    g = torch.Generator(device="cuda").manual_seed(3)
    B, H, L = 9, 3, 2200
    q = torch.randn(B, H, 64, generator=g, device="cuda").to(dtype)
    kc = torch.randn(B, H, L, 64, generator=g, device="cuda").to(dtype)
    vc = torch.randn(B, H, L, 64, generator=g, device="cuda").to(dtype)
    lengths = torch.tensor([0, 30, 511, 1022, 1023, 1024, 2000, L - 1, L + 5], device="cuda")
    out = glue.decode_attention(q, kc, vc, lengths).double()
    for b in range(B):
        n = int(lengths[b]) + 1
        if n > L:
            assert float(out[b].abs().max()) == 0.0
            continue
        s = torch.einsum("hd,hjd->hj", q[b].double(), kc[b, :, :n].double()) / 8.0
        ref = torch.einsum("hj,hjd->hd", torch.softmax(s, dim=-1), vc[b, :, :n].double())
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        assert float((out[b] - ref).abs().max()) <= tol * max(1.0, float(ref.abs().max())), b
