"""kdn_chunked_prefill_static: the exact prefill over the library's fixed scratch
array (no workspace argument, no allocation per call).

The GPU test checks two calls in a row (the second continuing the first's state,
on different tokens, so stale scratch would show) against kdn_chunked_prefill with
a caller workspace: the same kernels over the same scratch layout, so the results
must be bit-identical.  It also checks that a call rejected for its size leaves
the outputs untouched (nothing was enqueued) and that the second call takes no
device memory (no drop of a whole 2 MiB allocation granule in the device's free
memory; the test assumes no other process allocates on the GPU meanwhile).  The
CPU test checks the size limit.  This file is named to be collected last; it
passes alone as well.
"""

import ctypes

import numpy as np
import pytest
import torch

F32_TOL = 1e-4  # fp32-mode tolerance: max relative error per output row and on the state
DEV = "cuda:0"
KDN_STATIC_SCRATCH_BYTES = 64 * 1024 * 1024


def _rel(a, b):
    a = np.asarray(a, np.float64).reshape(-1, a.shape[-1])
    b = np.asarray(b, np.float64).reshape(-1, b.shape[-1])
    return float((np.linalg.norm(a - b, axis=-1) / np.maximum(np.linalg.norm(b, axis=-1), 1e-12)).max())


def _cpu_proj(D=512):
    from kdn_b200 import _lib

    p = _lib.KdnProjection()
    p.d_k, p.D, p.tau_inv, p.amp, p.phase = 64, D, 0.35, 0.0625, 8
    return p


def test_static_prefill_rejects_sizes_beyond_scratch():
    from kdn_b200 import _lib

    lib = _lib.load()
    p = _cpu_proj()

    def call(N, T, C=64):
        return lib.kdn_chunked_prefill_static(8, 8, 8, 0, 8, None, 0, None, 8, 0, 8, N, T, 64, C, p, None)

    need = lib.kdn_chunked_prefill_workspace_size(1, 20000, 64, 64, p, 0)
    assert need > KDN_STATIC_SCRATCH_BYTES
    assert call(1, 20000) == 4
    msg = lib.kdn_last_error()
    assert b"KDN_STATIC_SCRATCH_BYTES" in msg and str(need).encode() in msg
    assert call(16, 1024) == 4  # 16 x 1024 tokens: over the limit as well
    assert call(1, 1 << 40) == 4  # absurd T: rejected before any size arithmetic
    assert call(0, 64) == 1
    assert call(1, -1) == 1
    assert lib.kdn_chunked_prefill_workspace_size(4, 3000, 64, 64, p, 0) <= KDN_STATIC_SCRATCH_BYTES


def _inputs(seed, N, T, dv=64):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(N, T, 64, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(N, T, 64, generator=g), dim=-1)
    v = torch.randn(N, T, dv, generator=g)
    beta = torch.sigmoid(torch.randn(N, T, generator=g))
    decay = torch.sigmoid(torch.randn(N, T, generator=g) + 3)
    return [t.to(DEV) for t in (q, k, v, beta, decay)]


@pytest.mark.gpu
def test_static_prefill_matches_workspace_entry_two_calls():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import kdn_b200
    from kdn_b200 import _lib

    lib = _lib.load()
    proj = kdn_b200.FastWalshHadamardProjection(64, 512, 42).to(DEV)
    P, _keep = proj.kdn_projection(DEV)
    N, T, dv, C = 4, 1000, 64, 64  # ragged: 1000 = 15 chunks + 40 tokens
    stream = _lib.stream_handle(DEV)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr() if t is not None else None)
    segs = [_inputs(11, N, T, dv), _inputs(12, N, T, dv)]

    # the existing entry point with a caller workspace: two segments, state carried
    ws_bytes = int(lib.kdn_chunked_prefill_workspace_size(N, T, dv, C, P, _lib.KDN_MODE_F32))
    assert 0 < ws_bytes <= KDN_STATIC_SCRATCH_BYTES
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    ref_y, ref_s, s_in = [], [], None
    for q, k, v, beta, decay in segs:
        y = torch.empty(N, T, dv, device=DEV)
        s = torch.empty(N, dv, 512, device=DEV)
        rc = lib.kdn_chunked_prefill(ptr(q), ptr(k), ptr(v), 0, ptr(beta), ptr(decay), 0, ptr(s_in), ptr(y), 0,
                                     ptr(s), N, T, dv, C, P, _lib.KDN_MODE_F32, ptr(ws), ws_bytes, stream)
        assert rc == 0, lib.kdn_last_error()
        ref_y.append(y)
        ref_s.append(s)
        s_in = s
    torch.cuda.synchronize()

    # the static entry point: same two calls in a row, outputs allocated up front
    outs = [(torch.full((N, T, dv), float("nan"), device=DEV), torch.full((N, dv, 512), float("nan"), device=DEV))
            for _ in segs]
    free_after = []
    s_in = None
    for (q, k, v, beta, decay), (y, s) in zip(segs, outs):
        rc = lib.kdn_chunked_prefill_static(ptr(q), ptr(k), ptr(v), 0, ptr(beta), ptr(decay), 0, ptr(s_in), ptr(y),
                                            0, ptr(s), N, T, dv, C, P, stream)
        assert rc == 0, lib.kdn_last_error()
        torch.cuda.synchronize()
        free_after.append(torch.cuda.mem_get_info(0)[0])
        s_in = s
    assert free_after[0] - free_after[1] < 2 << 20, "the second call took device memory"

    for i in range(2):
        y, s = outs[i]
        assert torch.isfinite(y).all() and torch.isfinite(s).all()
        assert _rel(y.cpu().numpy(), ref_y[i].cpu().numpy()) <= F32_TOL
        assert _rel(s.cpu().numpy(), ref_s[i].cpu().numpy()) <= F32_TOL
        # same kernels, same scratch layout: stale scratch would break bit-equality
        assert torch.equal(y, ref_y[i]) and torch.equal(s, ref_s[i])

    # a call rejected for its size enqueues nothing: its outputs keep their contents
    big = [torch.zeros(4, 4096, 64, device=DEV) for _ in range(3)]
    bb = torch.zeros(4, 4096, device=DEV)
    yb = torch.full((4, 4096, dv), 7.0, device=DEV)
    sb = torch.full((4, dv, 512), 7.0, device=DEV)
    rc = lib.kdn_chunked_prefill_static(ptr(big[0]), ptr(big[1]), ptr(big[2]), 0, ptr(bb), None, 0, None, ptr(yb),
                                        0, ptr(sb), 4, 4096, dv, C, P, stream)
    assert rc == 4 and b"KDN_STATIC_SCRATCH_BYTES" in lib.kdn_last_error()
    torch.cuda.synchronize()
    assert bool((yb == 7.0).all()) and bool((sb == 7.0).all())
    code = ctypes.c_int(-1)
    assert lib.kdn_device_error(stream, ctypes.byref(code)) == 0 and code.value == 0
