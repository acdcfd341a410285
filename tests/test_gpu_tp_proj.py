"""Head-TP output projection with the all-reduce fused into the GEMM epilogue.

One rank: the kernel's product against a float32 torch product of the same bf16 operands
(tolerance 1e-4 relative to the largest output).  Two GPUs: every rank's result against
torch products summed by an NCCL all-reduce; the path must be the fused multicast one when
the GPUs are connected through NVSwitch with multicast, in all its forms (two-phase,
peer and one-shot), called repeatedly and alternately on one symmetric buffer.
"""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(300, 512, 128), (1024, 2048, 512), (4096, 256, 64)])
def test_local_projection_matches_torch(M, N, K):
    from kdn_b200 import distributed as kd

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    y = torch.randn(M, K, generator=g, device=dev).bfloat16()
    w = (torch.randn(N, K, generator=g, device=dev) / K ** 0.5).bfloat16()
    out, path = kd.row_parallel_out_proj(y, w)
    ref = y.float() @ w.float().t()
    torch.cuda.synchronize()
    assert path == "local"
    assert float((out - ref).abs().max() / ref.abs().max()) < 1e-4


def test_local_projection_bf16_output():
    from kdn_b200 import distributed as kd

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    y = torch.randn(777, 256, generator=g, device=dev).bfloat16()
    w = (torch.randn(768, 256, generator=g, device=dev) / 16).bfloat16()
    out, path = kd.row_parallel_out_proj(y, w, out_dtype=torch.bfloat16)
    ref = y.float() @ w.float().t()
    torch.cuda.synchronize()
    assert path == "local" and out.dtype == torch.bfloat16
    # one rounding of the fp32 product to bf16: within half an ulp (2^-9 relative)
    assert bool(((out.float() - ref).abs() <= ref.abs() * 2.0 ** -8 + 1e-6).all())


def test_fused_projection_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from test_distributed import _run
    import _dist_workers as W

    # 1100 rows: a partial last row of tiles (76 rows); 9 x 4 = 36 tiles over 2 owners
    for M, N, K in ((2048, 2048, 256), (1100, 1024, 128)):
        assert _run(W.nccl_tp_out_proj, 2, tmp_path, M, N, K) == ["ok", "ok"]
        paths = open(str(tmp_path / "result") + ".path").read().split(",")
        assert paths[:6] == ["fused-two-phase", "fused-one-shot", "fused-peer", "fused-two-phase", "fused-peer",
                             "fused-one-shot"], f"ran {paths}"
        assert paths[-2:] == ["fused-two-phase-bf16", "fused-peer-bf16"], f"ran {paths}"
