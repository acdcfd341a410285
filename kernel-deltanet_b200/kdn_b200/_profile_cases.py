"""Small, fixed invocations of single kernels for profiler captures (one call each, seeded inputs).

``python -m kdn_b200._profile_cases tp_proj``  -- the TMA-fed projection kernel, one rank, fp32 output:
    Y [32768, 512] bf16, W [2048, 512] bf16 -> [32768, 2048] fp32 (256 MiB out, above the L2 size).
``python -m kdn_b200._profile_cases decode_attn`` -- split-K decode attention, bf16 caches
    [8, 32, 16384, 64] (1 GiB of K and V), live lengths 4096..16383.
``python -m kdn_b200._profile_cases backward`` -- the prefill backward (exact fp32), 16 heads x 4096
    tokens, decay 1.
``python -m kdn_b200._profile_cases lift`` -- the standalone feature lift, 4 x 65536 unit vectors, bf16 in
    and out (32 MiB in, 256 MiB out).
Each case runs its call three times (two warm-ups, one to capture) and exits 0.
"""

from __future__ import annotations

import sys

import torch


def tp_proj():
    from .distributed import row_parallel_out_proj

    g = torch.Generator(device="cuda").manual_seed(0)
    y = torch.randn(32768, 512, generator=g, device="cuda").bfloat16()
    w = (torch.randn(2048, 512, generator=g, device="cuda") / 22.6).bfloat16()
    for _ in range(3):
        row_parallel_out_proj(y, w)
    torch.cuda.synchronize()


def decode_attn():
    from .kernels.glue import decode_attention

    g = torch.Generator(device="cuda").manual_seed(0)
    B, H, L = 8, 32, 16384
    q = torch.randn(B, H, 64, generator=g, device="cuda").bfloat16()
    kc = torch.randn(B, H, L, 64, generator=g, device="cuda").bfloat16()
    vc = torch.randn(B, H, L, 64, generator=g, device="cuda").bfloat16()
    lengths = torch.randint(4096, L, (B,), generator=g, device="cuda")
    for _ in range(3):
        decode_attention(q, kc, vc, lengths)
    torch.cuda.synchronize()


def lift():
    from .kernels.fwht import FastWalshHadamardProjection

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.nn.functional.normalize(torch.randn(4, 65536, 64, generator=g, device="cuda"), dim=-1).bfloat16()
    p = FastWalshHadamardProjection().to("cuda")
    for _ in range(3):
        p(x)
    torch.cuda.synchronize()


def backward():
    from .kernels.fused_kernel_deltanet import chunked_deltanet_backward
    from .kernels.fwht import FastWalshHadamardProjection

    g = torch.Generator(device="cuda").manual_seed(0)
    N, T = 16, 4096
    q = torch.nn.functional.normalize(torch.randn(N, T, 64, generator=g, device="cuda"), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(N, T, 64, generator=g, device="cuda"), dim=-1)
    v = torch.randn(N, T, 64, generator=g, device="cuda")
    beta = torch.sigmoid(torch.randn(N, T, generator=g, device="cuda"))
    dY = torch.randn(N, T, 64, generator=g, device="cuda")
    proj = FastWalshHadamardProjection().cuda()
    for _ in range(3):
        chunked_deltanet_backward(q, k, v, beta, None, dY, proj, 64)
    torch.cuda.synchronize()


if __name__ == "__main__":
    {"tp_proj": tp_proj, "decode_attn": decode_attn, "backward": backward, "lift": lift}[sys.argv[1]]()
    print("ok")
