"""Head-TP output projection with the all-reduce fused into the GEMM epilogue.

One rank: the kernel's product against a float32 torch product of the same bf16 operands
(tolerance 1e-4 relative to the largest output).  Two GPUs: every rank's result against
torch products summed by an NCCL all-reduce; the path must be the fused multicast one when
the GPUs are connected through NVSwitch with multicast.
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


def test_fused_projection_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from test_distributed import _run
    import _dist_workers as W

    assert _run(W.nccl_tp_out_proj, 2, tmp_path, 2048, 2048, 256) == ["ok", "ok"]
    path = open(str(tmp_path / "result") + ".path").read()
    assert path == "fused-multicast", f"ran the {path} path"
