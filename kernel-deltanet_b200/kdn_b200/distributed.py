"""Multi-GPU execution of the prefill: one process per GPU over torch.distributed.

Two ways to spread the work:

* Independent scans (data parallel).  The N = B*H scans of a layer share
  nothing, so each rank runs kdn prefill on its own contiguous share
  (``shard_range``) with no communication; a step ends when the slowest rank
  does (``max_over_ranks``).

* One long sequence over several ranks (sequence parallel).  Rank r holds the
  contiguous token block r of every scan.  The state map of a block is affine,
  S_out = S_in A_r + B_r (kernels/blelloch_scan.py:8-12), so:
    1. each rank forms its block's map (A_r [N, D, D], B_r [N, d_v, D]) in exact
       fp32 (``chunk_block_transition``);
    2. one all_gather shares the maps (1 MiB + 128 KiB per scan at D = 512);
    3. rank r folds the maps of ranks 0..r-1 onto the initial state -- the
       exclusive scan of the affine semigroup (kernels/blelloch_scan.py:42-56) --
       which gives the state entering its block;
    4. each rank runs its block's prefill from that state.
  The last rank's final state is the sequence's final state.  Remote data
  arrives through NCCL into local buffers; no kernel reads another GPU's memory.

The host orchestration (``entering_state``) takes the prefix fold as an argument
so that its rank logic runs under any backend; the library fold
(``kdn_affine_prefix_states``) is the default.

* Head tensor parallelism, output side (``row_parallel_out_proj``): rank r holds the
  scan outputs of its heads and its slice of the output projection; the layer output
  sum_r Y_r W_r^T is needed on every rank (serving/tensor_parallel_runner.py:51-75 runs a
  local GEMM, then an all-reduce).  One kernel (``kdn_tp_out_proj``) computes the tiles on
  the tensor cores and adds each into every rank's copy of a symmetric output buffer through
  its NVSwitch multicast address; a zeroing + barrier before and a barrier after (bounded,
  from torch's symmetric memory) frame it.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from .kernels.blelloch_scan import chunk_block_transition, prefix_states
from .kernels.fused_kernel_deltanet import fused_chunked_deltanet_forward
from .kernels.fwht import FastWalshHadamardProjection

PrefixFold = Callable[[torch.Tensor, torch.Tensor, Optional[torch.Tensor]], torch.Tensor]


def _world(group) -> Tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def shard_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous share [lo, hi) of n units for `rank` of `world`; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} rank={rank} world={world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def max_over_ranks(x: float, group=None, device: Optional[torch.device] = None) -> float:
    """Maximum of a host scalar over the ranks of `group` (a step time: the slowest rank)."""
    _, world = _world(group)
    if world == 1:
        return float(x)
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
            else torch.device("cpu")
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def kdn_prefix_fold(A: torch.Tensor, B: torch.Tensor, S0: Optional[torch.Tensor]) -> torch.Tensor:
    """S0 A[0] + B[0], then through every later map: the state after the last of the
    stacked maps A [m, N, D, D], B [m, N, d_v, D] (libkdn, exact fp32)."""
    _, final = prefix_states(A, B, S0, want_final=True)
    return final


def entering_state(A_local: torch.Tensor, B_local: torch.Tensor, initial_state: Optional[torch.Tensor],
                   group=None, fold: PrefixFold = kdn_prefix_fold) -> Optional[torch.Tensor]:
    """State entering this rank's block: every rank contributes its block map, rank r
    folds the maps of ranks 0..r-1 onto `initial_state` (None = zeros; it must be
    the same on every rank).  Rank 0 gets `initial_state` back unchanged."""
    rank, world = _world(group)
    if world == 1 or rank == 0:
        # every rank takes part in the same collective, rank 0 included
        if world > 1:
            _gather(A_local, B_local, group, world)
        return initial_state
    As, Bs = _gather(A_local, B_local, group, world)
    return fold(As[:rank], Bs[:rank], initial_state)


def _gather(A_local: torch.Tensor, B_local: torch.Tensor, group, world: int):
    """all_gather of every rank's (A, B) into stacked [world, ...] tensors (rank order)."""
    out = []
    for t in (A_local.contiguous(), B_local.contiguous()):
        stacked = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather(list(stacked.unbind(0)), t, group=group)
        out.append(stacked)
    return out[0], out[1]


def sequence_parallel_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                              decay: Optional[torch.Tensor], fwht_proj: FastWalshHadamardProjection,
                              chunk_size: int = 64, initial_state: Optional[torch.Tensor] = None, *,
                              group=None, mode: Optional[str] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Prefill of this rank's token block of one long sequence per scan.

    q, k [N, T_r, d_k], v [N, T_r, d_v], beta/decay [N, T_r] hold block r (blocks in
    rank order; lengths may differ).  Returns (y of the block [N, T_r, d_v], the
    state after the block [N, d_v, D]); on the last rank that state is the final
    state of the whole sequence.  The block maps are exact fp32; `mode` selects the
    arithmetic of the block prefill itself (as in fused_chunked_deltanet_forward).
    """
    _, world = _world(group)
    S_in = initial_state
    if world > 1:
        A, B = chunk_block_transition(k, v, beta, decay, fwht_proj, chunk_size)
        S_in = entering_state(A, B, initial_state, group)
    return fused_chunked_deltanet_forward(q, k, v, beta, decay, fwht_proj, chunk_size, S_in, mode=mode)


# ------------------------------------------------------------------ head-TP output projection
_SYMM: dict = {}
_BARRIER_TIMEOUT_MS = 60_000


def _symmetric_output(M: int, N: int, dev: torch.device, group):
    """A cached symmetric [M, N] fp32 buffer of `group` on `dev` and its handle."""
    import torch.distributed._symmetric_memory as symm_mem

    name = (group or dist.group.WORLD).group_name
    key = (M, N, dev.index, name)
    if key not in _SYMM:
        buf = symm_mem.empty(M, N, dtype=torch.float32, device=dev)
        hdl = symm_mem.rendezvous(buf, name)
        _SYMM[key] = (buf, hdl)
    return _SYMM[key]


def row_parallel_out_proj(y_local: torch.Tensor, w_local: torch.Tensor, group=None, *,
                          allow_unfused: bool = False) -> Tuple[torch.Tensor, str]:
    """sum over the ranks of `group` of y_local @ w_local^T, returned on every rank.

    y_local [M, K] and w_local [N, K] (bfloat16; K = local heads x d_v; N % 256 == 0,
    K % 64 == 0).  Returns (out [M, N] float32, path) with path "fused-multicast" (one
    kernel: tensor-core tiles reduced into every rank's copy through NVSwitch), "local"
    (one rank: the same kernel, stores) or, only when `allow_unfused` and the group has no
    multicast support, "unfused-nccl" (the kernel's product, then an NCCL all-reduce: the
    reference's two-step form).  The returned tensor of the fused path is the cached
    symmetric buffer: it is overwritten by the next call with the same shape.
    """
    from . import _lib

    if y_local.dim() != 2 or w_local.dim() != 2 or y_local.shape[1] != w_local.shape[1]:
        raise RuntimeError(f"expected y [M, K] and w [N, K]; got {tuple(y_local.shape)}, {tuple(w_local.shape)}")
    if not (y_local.is_cuda and w_local.is_cuda):
        raise RuntimeError("kdn_b200 runs on CUDA tensors only (no CPU fallback)")
    M, K = y_local.shape
    N = w_local.shape[0]
    dev = y_local.device
    y = y_local.to(torch.bfloat16).contiguous()
    w = w_local.to(torch.bfloat16).contiguous()
    lib = _lib.load()
    stream = _lib.stream_handle(dev)
    _, world = _world(group)
    if world == 1:
        out = torch.empty(M, N, device=dev, dtype=torch.float32)
        _lib.check(lib.kdn_tp_out_proj(y.data_ptr(), w.data_ptr(), out.data_ptr(), None, M, N, K, stream),
                   "kdn_tp_out_proj")
        return out, "local"
    from torch._C._autograd import DeviceType
    from torch._C._distributed_c10d import _SymmetricMemory

    buf, hdl = _symmetric_output(M, N, dev, group)
    if not _SymmetricMemory.has_multicast_support(DeviceType.CUDA, dev.index) or not hdl.multicast_ptr:
        if not allow_unfused:
            raise RuntimeError("no NVSwitch multicast for this group: the fused projection is unavailable "
                               "(pass allow_unfused=True for the GEMM + NCCL all-reduce form)")
        out = torch.empty(M, N, device=dev, dtype=torch.float32)
        _lib.check(lib.kdn_tp_out_proj(y.data_ptr(), w.data_ptr(), out.data_ptr(), None, M, N, K, stream),
                   "kdn_tp_out_proj")
        dist.all_reduce(out, group=group)
        return out, "unfused-nccl"
    buf.zero_()
    hdl.barrier(channel=0, timeout_ms=_BARRIER_TIMEOUT_MS)  # every copy is zero before anyone adds
    _lib.check(lib.kdn_tp_out_proj(y.data_ptr(), w.data_ptr(), None, hdl.multicast_ptr, M, N, K, stream),
               "kdn_tp_out_proj")
    hdl.barrier(channel=0, timeout_ms=_BARRIER_TIMEOUT_MS)  # every rank's tiles are in every copy
    return buf, "fused-multicast"


def release_symmetric_buffers() -> None:
    """Drop the cached symmetric output buffers (call before destroying the process group)."""
    _SYMM.clear()
