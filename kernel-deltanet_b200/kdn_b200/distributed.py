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
