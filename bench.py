"""Benchmark of the Kernel-DeltaNet hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...          (N > 1)

Workload: single-layer long-context prefill, B=1
sequence per GPU, H=16 heads, T=65536, d_k=64 lifted to D=512, d_v=64, chunk 64,
bf16 inputs, fp32 accumulation and state, zero initial state; q,k ~ N(0,1)
then L2-normalised, v ~ N(0,1), beta = sigmoid(N(0,1)), decay = 1.
A "step" is one prefill of that sequence.  With N GPUs every rank runs its own
sequence (whole sequences shard with no communication): weak scaling, value =
N * 65536 tokens / max-over-ranks step time.

The line also carries the decode workload (configs[3]: 64 streams x 16 heads,
fp32 state, one token per step) as ``decode`` and, on rank 0 at N=1, the CPU
baseline (the numpy port of the reference path, timed on a bounded sample).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import shutil
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "kernel-deltanet_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "KDN layer prefill tokens/s at T=64k,D=512 (1–8 B200); decode steps/s"

# Algorithmic work per chunk (64 tokens) of one sequence, per kernel of the two-phase
# tensor-core prefill (the path the library selects for fewer sequences than SMs):
#   chunk_prep : lift 2*128*64*512 + Gram 2*128*512*64 + U 2*64*64*64 FLOP; reads k,q,v
#                (bf16) and gates, writes the chunk record (U_q, U_k, T', U, Aq, factors)
#   state_pass : Y 2*64*512*64 + X 2*64*64*64 + update 2*512*64*64 FLOP; reads U_k, T', U,
#                factors, writes the entering state (fp16) and E
#   output_pass: 2*64*512*64 + 2*64*64*64 FLOP; reads U_q, state, E, Aq, writes y (bf16)
SPLIT_KERNELS = [
    ("chunk_prep_kernel", 2 * 128 * 64 * 512 + 2 * 128 * 512 * 64 + 2 * 64 ** 3,
     3 * 64 * 64 * 2 + 64 * 4 + 65536 * 2 + 8192 + 16384 + 8192 + 1024),
    ("state_pass_kernel", 2 * 64 * 512 * 64 + 2 * 64 ** 3 + 2 * 512 * 64 * 64,
     65536 + 8192 + 16384 + 1024 + 65536 + 8192),
    ("output_pass_kernel", 2 * 64 * 512 * 64 + 2 * 64 ** 3, 65536 + 65536 + 8192 + 8192 + 256 + 64 * 64 * 2),
]
B, H, T, DK, DV, D, C = 1, 16, 65536, 64, 64, 512, 64
FLOP_PER_TOKEN_HEAD = 360448  # 5 D-wide + 4 C-wide GEMMs per chunk / C (algorithmic count)
DEC_STREAMS, DEC_H = 64, 16
E2E_SEGMENT = 8192  # tokens per streamed segment of the end-to-end measurement
DEC_BYTES_PER_HEAD = 2 * DV * D * 4 + 3 * DK * 4 + 4 + DV * 4  # 263,172 B: state r+w, q,k,v, beta, y


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return {"hbm_gbs": j["hbm_gbs"], "bf16_tflops": j["bf16_tflops"],
                "bf16_tflops_sustained": j.get("bf16_tflops_sustained", j["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = f"/tmp/kdn_clocks_{os.getpid()}.csv"

    def _lines(self):
        try:
            with open(self.path) as f:
                return f.read().count("\n")
        except OSError:
            return 0

    def start(self):
        """Start sampling every 25 ms; returns once samples are flowing."""
        self.first = 0
        try:
            self.f = open(self.path, "w", buffering=1)
            cmd = ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                   "-lms", "25"]
            if shutil.which("stdbuf"):
                cmd = ["stdbuf", "-oL"] + cmd  # one line per sample, readable while it runs
            self.proc = subprocess.Popen(cmd, stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while self._lines() < 2 and time.time() - t0 < 10:
            time.sleep(0.02)

    def mark(self):
        """Call right before the timed region: later samples are the ones reported."""
        self.first = self._lines()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        last = self._lines()
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for i, line in enumerate(open(self.path)):
            if not (self.first <= i < last):
                continue
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, x in enumerate(r) if x.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(rows), "reasons": reasons}


def dist_init(backend):
    import datetime

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def prefill_inputs(dev, seed, n_heads=H, seq=T):
    import torch

    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(n_heads, seq, DK, generator=g, device=dev), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(n_heads, seq, DK, generator=g, device=dev), dim=-1)
    v = torch.randn(n_heads, seq, DV, generator=g, device=dev)
    beta = torch.sigmoid(torch.randn(n_heads, seq, generator=g, device=dev))
    return q.bfloat16(), k.bfloat16(), v.bfloat16(), beta


def cpu_inputs(n_heads: int, seq: int, seed: int = 0):
    """Seeded config-1 inputs on the host (float32): q, k unit vectors, v Gaussian, beta = sigmoid."""
    import torch

    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(n_heads, seq, DK, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(n_heads, seq, DK, generator=g), dim=-1)
    v = torch.randn(n_heads, seq, DV, generator=g)
    beta = torch.sigmoid(torch.randn(n_heads, seq, generator=g))
    return q, k, v, beta


def cpu_baseline(seq_sample: int, inputs=None):
    """The reference's CPU PyTorch prefill (fused_chunked_deltanet_forward with the dense-Omega lift,
    restated in torch: oracle/torch_chunked.py) on all host cores, one config-1 sequence of
    `seq_sample` tokens x 16 heads in float32."""
    import torch

    import oracle
    from oracle.torch_chunked import TorchProjection, chunked_forward

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    proj = TorchProjection(oracle.make_projection_constants())
    q, k, v, beta = inputs if inputs is not None else cpu_inputs(H, seq_sample)
    t0 = time.perf_counter()
    with torch.no_grad():
        chunked_forward(q, k, v, beta, None, proj, C)
    el = time.perf_counter() - t0
    return {"value": B * seq_sample / el, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"B=1 H={H} T={seq_sample}{' (config 1 in full)' if seq_sample == T else ''}: the "
                      f"reference's CPU torch path (kernels/fused_kernel_deltanet.py:31-155 with the dense lift "
                      f"of kernels/fwht.py:113-130, restated in oracle/torch_chunked.py), fp32, "
                      f"{torch.get_num_threads()} host threads, {el:.2f} s",
            "seconds": el}


def run_reference(args):
    """The reference arm: the reference's CPU PyTorch path on the host cores, config 1 (B=1, H=16,
    T=65536) per step; if one step takes longer than 12 s the later steps time the first half of the
    sequence instead (the path is linear in T, so tokens/s is unchanged), keeping the run bounded."""
    rank, world, _ = dist_init("gloo")
    if rank != 0:
        return
    seq = args.ref_seq
    inputs = cpu_inputs(H, seq)
    vals, samples = [], []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(seq, inputs)
        if i >= args.warmup:
            vals.append(r["value"])
            samples.append(seq)
        if r["seconds"] > 12.0 and seq > 4096:
            seq //= 2
            inputs = tuple(x[:, :seq].contiguous() for x in inputs)
    v = statistics.median(vals)
    r["value"] = v
    r["sample"] += f"; timed steps over T = {sorted(set(samples))}"
    r.pop("seconds", None)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * B * T / v,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"config1 prefill: B=1 seq, H={H}, T={T}, d_k={DK}->D={D}, d_v={DV}, C={C} "
                                   f"(CPU, host cores; ms_per_step scaled to T={T})", "global_batch": 1,
                       "seq_len": T, "heads": H, "parallelism": f"{r['cores']} host threads"},
            "cpu_baseline": r,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def bench_decode(dev, steps, warmup, peaks, rank=0, world=1):
    """Config 3: 64 streams x 16 heads, fp32 state, one token per stream per step, the streams
    sharded over the ranks (64 / world each, no communication).  A step is one token on every stream;
    steps/s = 1 / the slowest rank's step time."""
    import torch

    import kdn_b200
    from kdn_b200.distributed import max_over_ranks, shard_range

    lo, hi = shard_range(DEC_STREAMS, rank, world)
    ns = hi - lo
    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    states = 0.02 * torch.randn(ns, DEC_H, DV, D, generator=g, device=dev)
    n_in = min(steps + warmup, 64)  # token inputs cycle through 64 pre-drawn steps
    qs = torch.nn.functional.normalize(torch.randn(n_in, ns, DEC_H, DK, generator=g, device=dev), dim=-1)
    ks = torch.nn.functional.normalize(torch.randn(n_in, ns, DEC_H, DK, generator=g, device=dev), dim=-1)
    vs = torch.randn(n_in, ns, DEC_H, DV, generator=g, device=dev)
    bs = torch.sigmoid(torch.randn(n_in, ns, DEC_H, generator=g, device=dev))
    slots = torch.arange(ns, device=dev, dtype=torch.int64)
    out = torch.empty(ns, DEC_H, DV, device=dev)
    step = lambda i: kdn_b200.hybrid_recurrent_forward(qs[i % n_in], ks[i % n_in], vs[i % n_in], bs[i % n_in], None,
                                                       states, slots, out, fwht_proj=proj)
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(warmup, warmup + steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, device=dev)
    gbs = DEC_STREAMS * DEC_H * DEC_BYTES_PER_HEAD / (ms * 1e-3) / 1e9
    per_gpu_state = ns * DEC_H * DV * D * 4
    return {"metric": f"decode steps/s (64 streams x 16 heads, fp32 state 128 MiB, {ns} streams per GPU)",
            "value": 1e3 / ms, "unit": "steps/s", "ms_per_step": ms, "steps": steps, "streams_per_gpu": ns,
            "scaling": "strong",
            "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / world / peaks["hbm_gbs"], "traffic": None,
                         "note": f"per GPU; state {per_gpu_state / 2**20:.0f} MiB per GPU "
                                 f"({'fits in' if per_gpu_state < 120e6 else 'about'} the 126 MB L2); "
                                 f"peak {peaks['src']}"}}


# config 2: B=32 x H=16 = 512 independent scans of T=16384, sharded over the ranks
CFG2_SCANS, CFG2_T = 512, 16384


def bench_config2(dev, peaks, rank=0, world=1, steps=5, warmup=2):
    """Config 2: 512 (batch, head) scans x 16384 tokens, bf16 inputs, fp32 state; rank r takes a
    contiguous share of the scans (strong scaling, no communication).  tokens/s counts B*T = 32 x 16384
    tokens per step over the slowest rank's time; the roofline is the rank's prefill kernel against its
    share of the algorithmic FLOPs."""
    import torch

    import kdn_b200
    from kdn_b200.distributed import max_over_ranks, shard_range

    lo, hi = shard_range(CFG2_SCANS, rank, world)
    n = hi - lo
    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    q, k, v, beta = prefill_inputs(dev, 2000 + rank, n_heads=n, seq=CFG2_T)
    y = torch.empty(n, CFG2_T, DV, device=dev, dtype=torch.bfloat16)
    S = torch.empty(n, DV, D, device=dev, dtype=torch.float32)
    lib = kdn_b200.load()
    pstruct, _ = proj.kdn_projection(dev)
    ws_bytes = int(lib.kdn_chunked_prefill_workspace_size(n, CFG2_T, DV, C, pstruct, 1))
    ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    step = lambda: kdn_b200.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, C, mode="bf16", workspace=ws,
                                                           out=y, final_state=S)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms_local = e0.elapsed_time(e1) / steps
    ms = max_over_ranks(ms_local, device=dev)
    path = "split" if ws_bytes > 0 else "fused"
    tflops = FLOP_PER_TOKEN_HEAD * n * CFG2_T / (ms * 1e-3) / 1e12
    del q, k, v, beta, y, S, ws
    torch.cuda.empty_cache()
    return {"metric": "config2 batched prefill tokens/s (B=32 x H=16 = 512 scans, T=16384, bf16 in, fp32 state)",
            "value": 32 * CFG2_T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "scans_per_gpu": n, "scaling": "strong", "path": path,
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tflops / peaks["bf16_tflops"], "traffic": None,
                         "note": f"per GPU: {FLOP_PER_TOKEN_HEAD} FLOP/token-head x {n} x {CFG2_T} over the "
                                 f"slowest rank's step; {path} kernel path; peak {peaks['src']} burst"}}


def sp_error(dev, rank, world, n_heads=4, seq=16384):
    """Sequence-parallel prefill (row e2): rank r runs token block r of one sequence per head with the
    entering state folded from the other ranks' block maps (one NCCL all_gather); its block's outputs
    and the last rank's final state are compared with one single-GPU pass over the whole sequence
    (computed on every rank).  Returns the max over ranks of the relative errors (bf16 mode)."""
    import torch

    import kdn_b200
    from kdn_b200.distributed import max_over_ranks, sequence_parallel_prefill, shard_range

    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    q, k, v, beta = prefill_inputs(dev, 31337, n_heads=n_heads, seq=seq)
    Y, S = kdn_b200.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, C, mode="bf16")
    lo, hi = shard_range(seq // C, rank, world)
    a, b = lo * C, hi * C
    Yr, Sr = sequence_parallel_prefill(q[:, a:b].contiguous(), k[:, a:b].contiguous(), v[:, a:b].contiguous(),
                                       beta[:, a:b].contiguous(), None, proj, C, mode="bf16")
    ey = ((Yr.float() - Y[:, a:b].float()).norm(dim=-1) / Y[:, a:b].float().norm(dim=-1).clamp_min(1e-30)).max()
    es = ((Sr - S).norm() / S.norm()) if rank == world - 1 else torch.zeros((), device=dev)
    return {"y_block_vs_single_pass": max_over_ranks(float(ey), device=dev),
            "final_state_vs_single_pass": max_over_ranks(float(es), device=dev),
            "case": f"{n_heads} heads x {seq} tokens, bf16 mode, blocks of whole chunks per rank"}


def bench_lift(dev, peaks, steps=10, warmup=3):
    """The standalone feature lift (FastWalshHadamardProjection.forward -> kdn_fwht_lift) over config 1's
    q: 16 x 65536 unit-norm vectors, bf16 in and out.  HBM bound: 128 B read + 1 KiB written per vector
    (1.2 GB per call, larger than L2)."""
    import torch

    import kdn_b200

    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    x = prefill_inputs(dev, 7)[0]
    out = None
    for _ in range(warmup):
        out = proj(x)
    del out
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        out = proj(x)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    n = x.numel() // DK
    gbs = n * (DK + D) * 2 / (ms * 1e-3) / 1e9
    return {"metric": f"standalone feature lift vectors/s ({H} x {T} vectors, d_k {DK} -> D {D}, bf16 in/out)",
            "value": n / (ms * 1e-3), "unit": "vectors/s", "ms": ms, "steps": steps,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "traffic": None,
                         "note": f"{(DK + D) * 2} algorithmic bytes per vector; peak {peaks['src']}"}}


RAGGED_LENS = [128, 1024, 8192, 16384]  # the reference's ragged-batch example (serving/vllm_ragged_batching.py)


def bench_ragged(dev, steps, warmup):
    """Ragged prefill of four requests of different lengths x 16 heads over a slot pool (bf16 inputs)."""
    import torch

    import kdn_b200

    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    total = sum(RAGGED_LENS)
    g = torch.Generator(device=dev).manual_seed(11)
    q = torch.nn.functional.normalize(torch.randn(total, H, DK, generator=g, device=dev), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(total, H, DK, generator=g, device=dev), dim=-1).bfloat16()
    v = torch.randn(total, H, DV, generator=g, device=dev).bfloat16()
    beta = torch.sigmoid(torch.randn(total, H, generator=g, device=dev))
    cu = torch.tensor([0] + list(__import__("itertools").accumulate(RAGGED_LENS)), device=dev)
    pool = torch.zeros(8, H, DV, D, device=dev)
    slots = torch.tensor([5, 0, 3, 6], device=dev)
    out = torch.empty(total, H, DV, device=dev, dtype=torch.bfloat16)

    def step():
        kdn_b200.ragged_prefill(q, k, v, beta, None, cu, pool, slots, out, proj, mode="bf16")

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"metric": f"ragged prefill tokens/s ({len(RAGGED_LENS)} requests of {RAGGED_LENS} tokens x {H} heads, "
                      "slot pool, bf16)", "value": total / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
            "steps": steps}


# head-TP layer of the reference's TP benchmark (serving/tensor_parallel_runner.py:84-87): B=2, T=16384,
# d_model=2048, 16 heads x d_v=64, so the row-parallel output projection is [32768, 1024/world] x [1024/world, 2048]
TP_M, TP_N, TP_HEADS, TP_DV = 2 * 16384, 2048, 16, 64
NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool (nominal 900)


def bench_tp_out_proj(dev, rank, world, steps=10, warmup=3):
    """Row-parallel output projection + all-reduce over `world` GPUs: the fused kernel in both forms
    against the unfused forms (our GEMM + NCCL fp32 all-reduce; the reference's torch bf16 GEMM + NCCL
    bf16 all-reduce).  Every rank takes part; times are max over ranks."""
    import torch
    import torch.distributed as dist

    import kdn_b200
    from kdn_b200 import distributed as kd

    lib = kdn_b200.load()
    K = TP_HEADS * TP_DV // world
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    y = torch.randn(TP_M, K, generator=g, device=dev).bfloat16()
    w = (torch.randn(TP_N, K, generator=g, device=dev) / K ** 0.5).bfloat16()
    out32 = torch.empty(TP_M, TP_N, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def unfused():
        kdn_b200._lib.check(lib.kdn_tp_out_proj(y.data_ptr(), w.data_ptr(), out32.data_ptr(), 0, None, TP_M, TP_N,
                                                K, stream), "kdn_tp_out_proj")
        dist.all_reduce(out32)

    def reference_form():
        dist.all_reduce(y @ w.t())

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    res = {m: timed(lambda m=m: kd.row_parallel_out_proj(y, w, method=m)) for m in ("two-phase", "peer", "one-shot")}
    res["peer_bf16"] = timed(lambda: kd.row_parallel_out_proj(y, w, method="peer", out_dtype=torch.bfloat16))
    res["two-phase_bf16"] = timed(lambda: kd.row_parallel_out_proj(y, w, method="two-phase",
                                                                   out_dtype=torch.bfloat16))
    _, auto_path = kd.row_parallel_out_proj(y, w)
    res["unfused_nccl_fp32"] = timed(unfused)
    res["reference_torch_bf16_nccl"] = timed(reference_form)
    err = {}
    for m in ("two-phase", "peer", "peer_bf16", "two-phase_bf16"):
        fused, _ = kd.row_parallel_out_proj(y, w, method=m.replace("_bf16", ""),
                                            out_dtype=torch.bfloat16 if m.endswith("_bf16") else torch.float32)
        fused = fused.float()
        unfused()
        torch.cuda.synchronize()
        err[m] = float((fused - out32).abs().max() / out32.abs().max())
    kd.release_symmetric_buffers()
    method = auto_path.replace("fused-", "")
    out_bytes = TP_M * TP_N * 4
    # per GPU and direction: two-phase (1 + 1/w) B, peer 2 (w - 1)/w B, one-shot w B (into each GPU)
    link_bytes = out_bytes * {"two-phase": 1 + 1 / world, "peer": 2 * (world - 1) / world, "one-shot": world}[method]
    t_link = link_bytes / (NVLINK_GBS * 1e9) * 1e3
    t_tensor = 2 * TP_M * TP_N * K / (load_peaks()["bf16_tflops"] * 1e12) * 1e3
    ms = res[method]
    return {"metric": f"row-parallel out-proj + all-reduce ms ([{TP_M}, {K}] x [{K}, {TP_N}] per rank, fp32 sum)",
            "value": ms, "unit": "ms", "higher_is_better": False, "auto_path": auto_path, "ms": res,
            "max_rel_err_vs_nccl": err,
            "roofline": {"bound": "nvlink", "achieved": link_bytes / (ms * 1e-3) / 1e9, "peak": NVLINK_GBS,
                         "unit": "GB/s", "frac": max(t_link, t_tensor) / ms,
                         "note": f"{method} form (the auto choice): {link_bytes / out_bytes:.3f} x {out_bytes} B per "
                                 f"GPU and direction over NVLink "
                                 f"({t_link:.3f} ms at {NVLINK_GBS:.0f} GB/s measured peer copy) vs tensor "
                                 f"{t_tensor:.3f} ms; frac = max of both / measured"}}


# config 4: 22-block 20:2 hybrid LM, 64 sequences of lengths uniform in
# [4096, 65536] sharded over 8 GPUs (8 per GPU), ragged prefill then 256 greedy decode steps
LM_SEQS, LM_SEQS_PER_GPU, LM_DECODE_STEPS = 64, 8, 256


def bench_hybrid_lm(dev, rank, world, decode_steps=LM_DECODE_STEPS):
    """Per-GPU shard of config 4 through kdn_b200.models.KernelDeltaNetLM (bf16 weights and activations,
    tensor-core Kernel-DeltaNet prefill, fp32 recurrent state).  Rank r takes sequences [8r, 8r + 8) of the
    seeded 64 (mod 64 beyond 8 ranks).  Returns aggregate prefill and decode tokens/s (max time over ranks)."""
    import torch
    import torch.distributed as dist

    from kdn_b200.models import KernelDeltaNetLM

    torch.manual_seed(0)
    with torch.device(dev):
        model = KernelDeltaNetLM(mode="bf16")
    model = model.to(dev, torch.bfloat16).eval()
    g = torch.Generator().manual_seed(4242)
    lens_all = torch.randint(4096, 65537, (LM_SEQS,), generator=g).tolist()
    ids_all = [torch.randint(0, model.vocab_size, (n,), generator=g) for n in lens_all]
    pick = [(LM_SEQS_PER_GPU * rank + i) % LM_SEQS for i in range(LM_SEQS_PER_GPU)]
    lens = [lens_all[i] for i in pick]
    ids = torch.cat([ids_all[i] for i in pick]).to(dev)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    cache = model.new_cache(len(lens), max(lens) + decode_steps + 1)

    def timed(fn):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, r

    # warm-up: one untimed prefill of the same batch (library initialisation, allocator growth to the
    # workload's buffer sizes) and a few eager decode steps; the timed prefill then overwrites the cache
    model.prefill(ids, cu, cache)
    for _ in range(3):
        model.decode_step(torch.zeros(len(lens), dtype=torch.int64, device=dev), cache)
    pre_ms, logits = timed(lambda: model.prefill(ids, cu, cache))

    graph = model.capture_decode(cache, greedy=True)  # one decode step as a CUDA graph, argmax fed back
    graph.tokens.copy_(torch.argmax(logits, dim=-1))

    def decode():
        for _ in range(decode_steps):
            graph.step()
        return graph.tokens

    dec_ms, last = timed(decode)
    ok = bool(torch.isfinite(logits.float()).all()) and int(last.min()) >= 0
    del graph, cache, model
    torch.cuda.empty_cache()
    prompt_tokens = world * sum(lens)  # every rank holds a shard of the same size class
    return {"metric": "config4 20:2 hybrid LM (22 blocks, d_model 2048, 32x64 heads, SwiGLU 8192, vocab 32000, "
                      "anchors [10, 21]): ragged prefill tokens/s; greedy decode tokens/s",
            "prefill": {"value": world * sum(lens) / (pre_ms * 1e-3), "unit": "tokens/s", "ms": pre_ms,
                        "prompt_tokens_per_gpu": sum(lens)},
            "decode": {"value": world * len(lens) * decode_steps / (dec_ms * 1e-3), "unit": "tokens/s",
                       "ms_per_step": dec_ms / decode_steps, "steps": decode_steps},
            "sequences_per_gpu": len(lens), "lengths_rank0": lens if rank == 0 else None,
            "decode_note": "each step one CUDA-graph replay (22 layers + LM head + argmax); anchors use libkdn's "
                           "split-K decode attention over each sequence's live keys",
            "finite": ok, "dtype": "bf16 weights/activations, fp32 recurrent state",
            "data": "synthetic token ids (uniform over the vocab), random init", "prompt_tokens": prompt_tokens}


def run_lm_only(args):
    """Only the config-4 hybrid LM shard (any world size; torchrun for N > 1)."""
    import torch

    rank, world, local = dist_init("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    r = bench_hybrid_lm(dev, rank, world, decode_steps=args.lm_decode_steps)
    if rank == 0:
        print(json.dumps({"hybrid_lm": r, "n_gpus": world}), flush=True)


BWD_N, BWD_T = 16, 4096


def bench_backward(dev, steps=3):
    """The libkdn backward (exact fp32) of a [16 heads x 4096 tokens] prefill: dL/d(q, k, v, beta) for a
    given dL/dY (per rank; not a headline)."""
    import torch

    from kdn_b200 import FastWalshHadamardProjection, chunked_deltanet_backward

    proj = FastWalshHadamardProjection().to(dev)
    q, k, v, beta = (t.float() for t in prefill_inputs(dev, 99, n_heads=BWD_N, seq=BWD_T))
    dY = torch.randn(BWD_N, BWD_T, DV, device=dev, generator=torch.Generator(device=dev).manual_seed(5))
    chunked_deltanet_backward(q, k, v, beta, None, dY, proj, C)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        chunked_deltanet_backward(q, k, v, beta, None, dY, proj, C)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"metric": f"prefill backward token-heads/s ({BWD_N} heads x {BWD_T} tokens, exact fp32, per GPU)",
            "value": BWD_N * BWD_T / (ms * 1e-3), "unit": "token-heads/s", "ms": ms, "steps": steps}


def run_tp_proj_only(args):
    """Only the head-TP output projection comparison (world > 1 under torchrun)."""
    import torch

    rank, world, local = dist_init("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world < 2:
        raise SystemExit("--tp-proj-only needs 2 or more ranks (torchrun)")
    r = bench_tp_out_proj(dev, rank, world, steps=args.steps, warmup=args.warmup)
    if rank == 0:
        print(json.dumps({"tp_out_proj": r, "n_gpus": world}), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    import kdn_b200

    rank, world, local = dist_init("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    peaks = load_peaks()
    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    q, k, v, beta = prefill_inputs(dev, 1234 + rank)
    y = torch.empty(H, T, DV, device=dev, dtype=torch.bfloat16)
    S = torch.empty(H, DV, D, device=dev, dtype=torch.float32)
    lib = kdn_b200.load()
    pstruct, _ = proj.kdn_projection(dev)
    ws_bytes = int(lib.kdn_chunked_prefill_workspace_size(H, T, DV, C, pstruct, 1))
    ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)

    def step(qq=q, kk=k, vv=v, bb=beta):
        kdn_b200.fused_chunked_deltanet_forward(qq, kk, vv, bb, None, proj, C, mode="bf16", workspace=ws, out=y,
                                                final_state=S)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # per-launch events, recorded by the library on the launch stream inside the timed region
    nmarks = 8
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(nmarks)] for _ in range(args.steps)]
    for row in marks:
        for ev in row:
            ev.record()  # creates the CUDA event
    handles = [(ctypes.c_void_p * nmarks)(*[ev.cuda_event for ev in row]) for row in marks]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(2):  # keep the GPU busy while the sampler starts
        step()
    torch.cuda.synchronize()
    clocks.mark()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        lib.kdn_set_prefill_events(handles[i], nmarks)
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    clk = clocks.stop()
    nlaunch = int(lib.kdn_prefill_launch_count())
    launch_ms = [statistics.mean(marks[i][j].elapsed_time(marks[i][j + 1]) for i in range(args.steps))
                 for j in range(min(nlaunch, nmarks - 1))]
    if world > 1:
        dist.barrier()
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # end to end through the public API: pinned host inputs in, host outputs back; the call streams the
    # sequence through the GPU in segments (host->device copies, kernels and device->host copies overlap)
    hq, hk, hv, hb = (x.cpu().pin_memory() for x in (q, k, v, beta))
    hy = torch.empty(y.shape, dtype=y.dtype).pin_memory()
    hS = torch.empty(S.shape, dtype=S.dtype).pin_memory()
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, hb))
    d2h = hy.numel() * hy.element_size() + hS.numel() * hS.element_size()

    def e2e_step():
        kdn_b200.fused_chunked_deltanet_forward(hq, hk, hv, hb, None, proj, C, mode="bf16", out=hy, final_state=hS,
                                                device=dev, segment_tokens=args.e2e_segment)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_steps = max(3, min(args.steps, 10))
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    dec = bench_decode(dev, steps=1024, warmup=5, peaks=peaks, rank=rank, world=world)
    cfg2 = bench_config2(dev, peaks, rank, world)
    lift = bench_lift(dev, peaks)
    rag = bench_ragged(dev, steps=10, warmup=3)
    tpp = bench_tp_out_proj(dev, rank, world) if world > 1 else None
    sp = sp_error(dev, rank, world) if world > 1 else None
    bwd = bench_backward(dev)
    lm = bench_hybrid_lm(dev, rank, world) if not args.no_lm else None

    if world > 1:
        dist.barrier()
    if rank != 0:
        return
    tokens = world * B * T
    flops = FLOP_PER_TOKEN_HEAD * B * H * T
    traffic_db = {}
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        traffic_db = json.load(open(tp))
    chunks = B * H * ((T + C - 1) // C)
    if nlaunch == len(SPLIT_KERNELS):
        j = max(range(nlaunch), key=lambda i: launch_ms[i])
        kname, kflop, kbytes = SPLIT_KERNELS[j]
        k_ms = launch_ms[j]
        kflops, kb = kflop * chunks, kbytes * chunks
        t_frac = kflops / (k_ms * 1e-3) / 1e12 / peaks["bf16_tflops"]
        h_frac = kb / (k_ms * 1e-3) / 1e9 / peaks["hbm_gbs"]
        kinfo = traffic_db.get(kname, {})
        if h_frac >= t_frac:
            roof = {"bound": "hbm", "achieved": kb / (k_ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": h_frac}
        else:
            roof = {"bound": "tensor", "achieved": kflops / (k_ms * 1e-3) / 1e12, "peak": peaks["bf16_tflops"],
                    "unit": "TFLOP/s", "frac": t_frac}
        roof["traffic"] = kinfo.get("bytes_per_launch")
        roof["kernel"] = kname
        roof["kernel_ms"] = k_ms
        roof["note"] = (f"dominant kernel of {nlaunch} launches per step (ms each: "
                        f"{', '.join(f'{SPLIT_KERNELS[i][0]} {launch_ms[i]:.3f}' for i in range(nlaunch))}); "
                        f"algorithmic {kflop} FLOP and {kbytes} B per chunk-sequence x {chunks} chunks; "
                        f"tensor {t_frac:.3f} / hbm {h_frac:.3f} of {peaks['src']} peaks (burst); the state "
                        f"pass is a serial chain per sequence (latency bound); whole step "
                        f"{flops / (ms * 1e-3) / 1e12:.1f} TFLOP/s algorithmic")
    else:
        # one launch does the whole prefill: the persistent two-phase kernel when the library needs a
        # workspace for this shape (fewer sequences than SMs), else the fused one-CTA-per-sequence kernel
        kname = "split_persistent_kernel" if ws_bytes > 0 else "prefill_tc_kernel"
        k_ms = launch_ms[0] if launch_ms else ms
        achieved = flops / (k_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"],
                "traffic": traffic_db.get(kname, {}).get("bytes_per_launch"), "kernel": kname, "kernel_ms": k_ms,
                "note": f"{kname}: the whole prefill in {nlaunch} launch(es); algorithmic {FLOP_PER_TOKEN_HEAD} "
                        f"FLOP/token-head x {B * H * T} token-heads; peak {peaks['src']} burst; HBM traffic "
                        f"{(traffic_db.get(kname, {}).get('bytes_per_launch') or 0) / (k_ms * 1e-3) / 1e9:.0f} "
                        f"GB/s of {peaks['hbm_gbs']:.0f}"}
    launches_per_step = nlaunch
    line = {
        "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"config1 prefill: B=1 seq per GPU, H={H}, T={T}, d_k={DK}->D={D}, d_v={DV}, C={C}, "
                               "bf16 in, fp32 accumulate/state", "global_batch": world * B, "seq_len": T,
                   "heads": H, "parallelism": f"dp{world} (whole sequences per rank, no communication)",
                   "l2": "inputs 402 MB per step > 126 MB L2 (no flush needed)"},
        "roofline": roof,
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
        "decode": dec,
        "config2": cfg2,
        "lift": lift,
        "ragged": rag,
    }
    if tpp is not None:
        line["tp_out_proj"] = tpp
    if sp is not None:
        line["sequence_parallel"] = sp
    line["backward"] = bwd
    if lm is not None:
        line["hybrid_lm"] = lm
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.ref_seq)
        line["cpu_baseline"].pop("seconds", None)
    print(json.dumps(line), flush=True)


def run_prefill_only(n_seq: int, seq: int, mode: str = "bf16"):
    """Two prefill calls on seeded inputs of [n_seq, seq] (the case `ncu` captures use); mode "fp32" runs
    the exact CUDA-core path on fp32 copies of the inputs."""
    import torch

    import kdn_b200

    dev = torch.device("cuda", 0)
    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    q, k, v, beta = prefill_inputs(dev, 7, n_heads=n_seq, seq=seq)
    dt = torch.float32 if mode == "fp32" else torch.bfloat16
    q, k, v = (t.to(dt) for t in (q, k, v))
    y = torch.empty(n_seq, seq, DV, device=dev, dtype=dt)
    S = torch.empty(n_seq, DV, D, device=dev, dtype=torch.float32)
    for _ in range(2):
        kdn_b200.fused_chunked_deltanet_forward(q, k, v, beta, None, proj, C, mode=mode, out=y, final_state=S)
    torch.cuda.synchronize()
    print(json.dumps({"prefill_only": [n_seq, seq], "launches_per_call": int(kdn_b200.load().kdn_prefill_launch_count()),
                      "path": os.environ.get("KDN_PREFILL_PATH", "auto")}))


def run_case(name: str):
    """One fixed, seeded invocation of a single kernel, three calls (two warm-ups, one to capture), for
    profiler captures of kernels outside the headline step:
      tp_proj      the TMA-fed projection kernel, one rank: Y [32768, 512] x W [2048, 512]^T, bf16 -> fp32
      decode_attn  split-K decode attention, bf16 caches [8, 32, 16384, 64], live lengths 4096..16383
      backward     the prefill backward (exact fp32), 16 heads x 4096 tokens, decay 1
      lift         the standalone feature lift, 4 x 65536 unit vectors, bf16 in and out
      anchor_attn  the anchors' varlen causal attention, 4 sequences x 8192 tokens x 32 heads (bf16)
      lm           the config-4 LM (22 blocks, random init): a prefill of 2 sequences (4096 + 8192 tokens)
                   and 2 eager decode steps (every LM kernel, for a launch list)"""
    import torch

    import kdn_b200

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    if name == "tp_proj":
        from kdn_b200.distributed import row_parallel_out_proj

        y = torch.randn(32768, 512, generator=g, device=dev).bfloat16()
        w = (torch.randn(2048, 512, generator=g, device=dev) / 22.6).bfloat16()
        call = lambda: row_parallel_out_proj(y, w)
    elif name == "decode_attn":
        from kdn_b200.kernels.glue import decode_attention

        Bq, Hq, L = 8, 32, 16384
        q = torch.randn(Bq, Hq, 64, generator=g, device=dev).bfloat16()
        kc = torch.randn(Bq, Hq, L, 64, generator=g, device=dev).bfloat16()
        vc = torch.randn(Bq, Hq, L, 64, generator=g, device=dev).bfloat16()
        lengths = torch.randint(4096, L, (Bq,), generator=g, device=dev)
        call = lambda: decode_attention(q, kc, vc, lengths)
    elif name == "lift":
        x = torch.nn.functional.normalize(torch.randn(4, 65536, 64, generator=g, device=dev), dim=-1).bfloat16()
        p = kdn_b200.FastWalshHadamardProjection().to(dev)
        call = lambda: p(x)
    elif name == "anchor_attn":
        from kdn_b200.kernels.glue import varlen_causal_attention

        Ha, La, Ba = 32, 8192, 4
        n = Ba * La
        q = torch.randn(Ha, n, 64, generator=g, device=dev).bfloat16()
        kc = torch.randn(Ba, Ha, La, 64, generator=g, device=dev).bfloat16()
        vc = torch.randn(Ba, Ha, La, 64, generator=g, device=dev).bfloat16()
        cu = torch.arange(0, n + 1, La, device=dev, dtype=torch.int64)
        call = lambda: varlen_causal_attention(q, kc, vc, cu, La)
    elif name == "lm":
        from kdn_b200.models import KernelDeltaNetLM

        torch.manual_seed(0)
        with torch.device(dev):
            model = KernelDeltaNetLM(mode="bf16")
        model = model.to(dev, torch.bfloat16).eval()
        lens = [4096, 8192]
        ids = torch.randint(0, model.vocab_size, (sum(lens),), generator=g, device=dev)
        cache = model.new_cache(len(lens), max(lens) + 8)

        def call():
            model.prefill(ids, [0, lens[0], sum(lens)], cache)
            for _ in range(2):
                model.decode_step(torch.zeros(len(lens), dtype=torch.int64, device=dev), cache)
    elif name == "backward":
        Nb, Tb = 16, 4096
        q = torch.nn.functional.normalize(torch.randn(Nb, Tb, 64, generator=g, device=dev), dim=-1)
        k = torch.nn.functional.normalize(torch.randn(Nb, Tb, 64, generator=g, device=dev), dim=-1)
        v = torch.randn(Nb, Tb, 64, generator=g, device=dev)
        beta = torch.sigmoid(torch.randn(Nb, Tb, generator=g, device=dev))
        dY = torch.randn(Nb, Tb, 64, generator=g, device=dev)
        proj = kdn_b200.FastWalshHadamardProjection().to(dev)
        call = lambda: kdn_b200.chunked_deltanet_backward(q, k, v, beta, None, dY, proj, 64)
    else:
        raise SystemExit(f"unknown case {name!r}")
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    print(json.dumps({"case": name, "ok": True}))


def run_decode_only(steps: int):
    """Only the decode workload for `steps` steps (the case `ncu` captures use)."""
    import torch

    dev = torch.device("cuda", 0)
    r = bench_decode(dev, steps=steps, warmup=3, peaks=load_peaks())
    torch.cuda.synchronize()
    print(json.dumps({"decode_only": steps, "ms_per_step": r["ms_per_step"], "gbs": r["roofline"]["achieved"]}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-seq", type=int, default=T, help="tokens per CPU-baseline sample (16 heads)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill-only", type=int, nargs=2, metavar=("N", "T"),
                    help="only run two prefill calls of N sequences x T tokens (for profiler captures)")
    ap.add_argument("--prefill-mode", default="bf16", choices=["bf16", "fp32"],
                    help="arithmetic mode of --prefill-only")
    ap.add_argument("--case", choices=["tp_proj", "decode_attn", "backward", "lift", "anchor_attn", "lm"],
                    help="only run one fixed single-kernel invocation three times (for profiler captures)")
    ap.add_argument("--decode-only", type=int, metavar="STEPS",
                    help="only run the decode workload for STEPS steps (for profiler captures)")
    ap.add_argument("--lm-only", action="store_true", help="only run the config-4 hybrid LM shard")
    ap.add_argument("--no-lm", action="store_true", help="skip the config-4 hybrid LM shard in the full run")
    ap.add_argument("--e2e-segment", type=int, default=E2E_SEGMENT, help="tokens per streamed segment (e2e)")
    ap.add_argument("--lm-decode-steps", type=int, default=LM_DECODE_STEPS)
    ap.add_argument("--tp-proj-only", action="store_true",
                    help="only compare the head-TP output projection forms (2+ ranks under torchrun)")
    args = ap.parse_args()
    if args.lm_only:
        run_lm_only(args)
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()
        return
    if args.tp_proj_only:
        run_tp_proj_only(args)
        import torch.distributed as dist

        dist.destroy_process_group()
        return
    if args.case:
        run_case(args.case)
        return
    if args.decode_only:
        run_decode_only(args.decode_only)
        return
    if args.prefill_only:
        run_prefill_only(*args.prefill_only, mode=args.prefill_mode)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)
    try:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()
    except Exception:
        pass


if __name__ == "__main__":
    main()
