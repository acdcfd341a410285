"""Rank bodies for the multi-process tests (spawned; one process per rank).

CPU (gloo) workers exercise the host orchestration of kdn_b200.distributed with
the block maps and the fold computed by the oracle / torch on the host -- the
product's own fold is the libkdn kernel, checked by the GPU tests.  The NCCL
worker runs the whole sequence-parallel prefill through libkdn on one GPU per rank.
"""

from __future__ import annotations

import datetime
import os
import sys
import traceback

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for _p in (ROOT, os.path.join(ROOT, "kernel-deltanet_b200"), HERE):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def _init(rank, world, port, backend):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    return dist


def sequence_inputs(seed, N, T, dv=64):
    import numpy as np

    rng = np.random.default_rng(seed)
    q = rng.standard_normal((N, T, 64)); q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((N, T, 64)); k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((N, T, dv))
    beta = 1 / (1 + np.exp(-rng.standard_normal((N, T))))
    decay = 1 / (1 + np.exp(-(rng.standard_normal((N, T)) + 3)))
    S0 = 0.1 * rng.standard_normal((N, dv, 512))
    return q, k, v, beta, decay, S0


def block_bounds(T, world):
    """Ragged blocks on purpose: rank r gets a share that is not a multiple of the chunk."""
    cuts = [0] + [int(T * (r + 1) / world) + (7 if r + 1 < world else 0) for r in range(world)]
    cuts[-1] = T
    return cuts


def gloo_sequence_parallel(rank, world, port, result_path):
    """entering_state + block prefill per rank vs the oracle's single pass (all fp64 on the host)."""
    ok = False
    try:
        import numpy as np
        import torch

        import oracle
        from kdn_b200 import distributed as kd

        dist = _init(rank, world, port, "gloo")
        c = oracle.make_projection_constants()
        N, T = 2, 200
        q, k, v, beta, decay, S0 = sequence_inputs(11, N, T)
        y_full, S_full = oracle.chunked_deltanet_forward(q, k, v, beta, decay, c, 32, S0)
        cuts = block_bounds(T, world)
        lo, hi = cuts[rank], cuts[rank + 1]
        blk = lambda a: a[:, lo:hi]
        A, B = oracle.chunk_block_transition(blk(q), blk(k), blk(v), blk(beta), blk(decay), c, 32)

        def host_fold(As, Bs, S):
            S = torch.zeros_like(Bs[0]) if S is None else S
            for a, b in zip(As.unbind(0), Bs.unbind(0)):
                S = S @ a + b
            return S

        S_in = kd.entering_state(torch.from_numpy(A), torch.from_numpy(B), torch.from_numpy(S0), fold=host_fold)
        y, S_out = oracle.chunked_deltanet_forward(blk(q), blk(k), blk(v), blk(beta), blk(decay), c, 32,
                                                   S_in.numpy())
        err_y = np.abs(y - y_full[:, lo:hi]).max() / np.abs(y_full).max()
        # the state after block r is the full scan's state after token hi
        _, S_ref = oracle.chunked_deltanet_forward(q[:, :hi], k[:, :hi], v[:, :hi], beta[:, :hi], decay[:, :hi],
                                                   c, 32, S0)
        err_s = np.abs(S_out - S_ref).max() / np.abs(S_ref).max()
        if rank == world - 1:
            err_s = max(err_s, np.abs(S_out - S_full).max() / np.abs(S_full).max())
        t = kd.max_over_ranks(rank + 0.5)
        lo_s, hi_s = kd.shard_range(37, rank, world)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([hi_s - lo_s]))
        ok = (err_y < 1e-10 and err_s < 1e-10 and t == world - 0.5 and sum(int(s) for s in sizes) == 37)
        if not ok:
            print(f"rank {rank}: err_y {err_y} err_s {err_s} max {t} sizes {sizes}", flush=True)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        traceback.print_exc()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write("ok" if ok else "fail")


def nccl_sequence_parallel(rank, world, port, result_path, mode):
    """sequence_parallel_prefill through libkdn, one GPU per rank, vs the oracle."""
    ok = False
    try:
        import numpy as np
        import torch

        import oracle
        from kdn_b200 import distributed as kd
        import kdn_b200

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist = _init(rank, world, port, "nccl")
        c = oracle.make_projection_constants()
        N, T = 2, 520
        q, k, v, beta, decay, S0 = sequence_inputs(21, N, T)
        dt = torch.bfloat16 if mode == "bf16" else torch.float32
        if mode == "bf16":  # the oracle runs on the rounded inputs
            q, k, v = (torch.from_numpy(a).bfloat16().double().numpy() for a in (q, k, v))
        y_full, S_full = oracle.chunked_deltanet_forward(q, k, v, beta, decay, c, 64, S0)
        cuts = block_bounds(T, world)
        lo, hi = cuts[rank], cuts[rank + 1]
        g = lambda a, d=torch.float32: torch.from_numpy(np.ascontiguousarray(a[:, lo:hi])).to(dev, d)
        proj = kdn_b200.FastWalshHadamardProjection().to(dev)
        y, S = kd.sequence_parallel_prefill(g(q, dt), g(k, dt), g(v, dt), g(beta), g(decay), proj, 64,
                                            torch.from_numpy(S0).float().to(dev), mode=mode)
        torch.cuda.synchronize()
        y = y.float().cpu().numpy()
        ref = y_full[:, lo:hi]
        err_y = float(np.max(np.linalg.norm(y - ref, axis=-1) / np.maximum(np.linalg.norm(ref, axis=-1), 1e-30)))
        tol_y, tol_s = (2e-2, 1e-2) if mode == "bf16" else (1e-4, 1e-4)
        ok = err_y < tol_y
        if rank == world - 1:
            S = S.cpu().numpy()
            err_s = float(np.linalg.norm(S - S_full) / np.linalg.norm(S_full))
            ok = ok and err_s < tol_s
        else:
            err_s = None
        print(f"rank {rank} mode {mode}: err_y {err_y:.3e} err_s {err_s}", flush=True)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        traceback.print_exc()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write("ok" if ok else "fail")


def nccl_tp_out_proj(rank, world, port, result_path, M, N, K):
    """row_parallel_out_proj (fused multicast reduction) vs torch matmuls + NCCL all-reduce."""
    ok = False
    try:
        import torch

        from kdn_b200 import distributed as kd

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist = _init(rank, world, port, "nccl")
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        y = torch.randn(M, K, generator=g, device=dev).bfloat16()
        w = (torch.randn(N, K, generator=g, device=dev) / K ** 0.5).bfloat16()
        ref = y.float() @ w.float().t()
        dist.all_reduce(ref)
        paths, errs = [], []
        # repeated and alternating calls reuse one symmetric buffer and its tile counters
        for method in ("two-phase", "one-shot", "peer", "two-phase", "peer", "one-shot", "auto"):
            out, path = kd.row_parallel_out_proj(y, w, method=method, allow_unfused=True)
            torch.cuda.synchronize()
            errs.append(float((out - ref).abs().max() / ref.abs().max()))
            paths.append(path)
        err_bf16 = 0.0
        for method in ("two-phase", "auto"):  # the switch's fp32 sum of bf16 copies, then peer (auto at world 2)
            out, path = kd.row_parallel_out_proj(y, w, method=method, out_dtype=torch.bfloat16)
            torch.cuda.synchronize()
            err_bf16 = max(err_bf16, float((out.float() - ref).abs().max() / ref.abs().max()))
            paths.append(path + "-bf16")
        same = torch.tensor([float(out.float().sum())], device=dev, dtype=torch.float64)
        everyone = [torch.zeros_like(same) for _ in range(world)]
        dist.all_gather(everyone, same)  # the owner's sum is copied: every rank holds the same bits
        ok = (max(errs) < 1e-4 and err_bf16 < 1e-2 and all(float(e) == float(same) for e in everyone)
              and all(p.startswith("fused-") or p == "unfused-nccl" for p in paths[:-1]))
        print(f"rank {rank}: paths {paths} errs {[f'{e:.1e}' for e in errs]} bf16 {err_bf16:.1e}", flush=True)
        with open(f"{result_path}.path", "w") as f:
            f.write(",".join(paths))
        kd.release_symmetric_buffers()
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        traceback.print_exc()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write("ok" if ok else "fail")
