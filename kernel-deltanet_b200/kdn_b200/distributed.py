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
ONE_SHOT_MAX_BYTES = 2 << 20  # "auto" picks the one-shot form up to this output size


class _SymmetricOutput:
    """A symmetric allocation of `group` holding the [M, N] output (fp32 or bf16) and, behind
    it, one uint32 counter per output tile (zeroed once, at creation, on every rank)."""

    def __init__(self, M: int, N: int, dtype: torch.dtype, dev: torch.device, group, lib):
        import torch.distributed._symmetric_memory as symm_mem

        name = (group or dist.group.WORLD).group_name
        esize = torch.empty((), dtype=dtype).element_size()
        self.tiles = int(lib.kdn_tp_out_proj_tiles(M, N))
        self.ctr_off = (M * N * esize + 15) // 16 * 16  # byte offset of the counters (16-byte aligned)
        self.raw = symm_mem.empty(self.ctr_off + 4 * self.tiles, dtype=torch.uint8, device=dev)
        self.hdl = symm_mem.rendezvous(self.raw, name)
        self.out = self.raw[:M * N * esize].view(dtype).view(M, N)
        self.counters = self.raw[self.ctr_off:].view(torch.int32)
        self.counters.zero_()
        self.calls = 0  # owner-scheme calls made on this buffer: the counters reach calls * world
        self.hdl.barrier(channel=0, timeout_ms=_BARRIER_TIMEOUT_MS)

    def multicast(self, byte_offset: int = 0) -> int:
        return int(self.hdl.multicast_ptr) + byte_offset

    def peer_ptrs(self, byte_offset: int = 0):
        """Every rank's copy (rank order), mapped into this process, at a byte offset."""
        return [int(p) + byte_offset for p in self.hdl.buffer_ptrs]


def _symmetric_output(M: int, N: int, dtype: torch.dtype, dev: torch.device, group, lib) -> _SymmetricOutput:
    key = (M, N, dtype, dev.index, (group or dist.group.WORLD).group_name)
    if key not in _SYMM:
        _SYMM[key] = _SymmetricOutput(M, N, dtype, dev, group, lib)
    return _SYMM[key]


def row_parallel_out_proj(y_local: torch.Tensor, w_local: torch.Tensor, group=None, *, method: str = "auto",
                          out_dtype: torch.dtype = torch.float32,
                          allow_unfused: bool = False) -> Tuple[torch.Tensor, str]:
    """sum over the ranks of `group` of y_local @ w_local^T, returned on every rank.

    y_local [M, K] and w_local [N, K] (bfloat16; K = local heads x d_v; N % 256 == 0,
    K % 64 == 0).  Returns (out [M, N] float32, path).  With one rank the kernel stores its
    product (path "local").  Otherwise one kernel computes the tiles on the tensor cores and
    reduces them across the ranks (path "fused-<method>"):
      * "two-phase": every rank stores its tiles locally and announces them; the owner of each
        tile sums all copies in the NVSwitch (multimem.ld_reduce, fp32 accumulation for bf16
        copies too) and writes the sum to every copy (multimem.st): (1 + 1/world) x the output
        bytes cross each GPU's links;
      * "peer": the same owner scheme over peer pointers (loads from every copy, stores into
        every copy): 2 (world - 1) / world x the output bytes, fewer than two-phase at world 2,
        and no multicast needed;
      * "one-shot": each tile is added into every copy through the multicast address as it is
        produced (one pass, world x the output bytes into each GPU);
      * "auto": peer at world 2 (or without multicast), else two-phase -- and for fp32 outputs up
        to ONE_SHOT_MAX_BYTES, one-shot.
    The sum is formed in fp32 and is identical on every rank.  out_dtype torch.bfloat16 (the
    reference's layer dtype; every method but one-shot): every rank's product is rounded to bf16
    once and the sum once, and half the bytes move.  Only when `allow_unfused` and the group
    cannot map symmetric memory: the kernel's product and then an NCCL all-reduce (path
    "unfused-nccl", the reference's two-step form).  The tensor returned by a fused path is a
    cached symmetric buffer, overwritten by the next call with the same shape.
    """
    import ctypes

    from . import _lib

    if method not in ("auto", "one-shot", "two-phase", "peer"):
        raise ValueError(f"method must be 'auto', 'one-shot', 'two-phase' or 'peer', got {method!r}")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"out_dtype must be torch.float32 or torch.bfloat16, got {out_dtype}")
    if out_dtype == torch.bfloat16 and method == "one-shot":
        raise ValueError("the one-shot method adds into the fp32 output; bf16 output takes 'two-phase' or 'peer'")
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
    rank, world = _world(group)

    def local_product():
        out = torch.empty(M, N, device=dev, dtype=out_dtype)
        _lib.check(lib.kdn_tp_out_proj(y.data_ptr(), w.data_ptr(), out.data_ptr(), _lib.dtype_code(out), None, M, N,
                                       K, stream), "kdn_tp_out_proj")
        return out

    if world == 1:
        return local_product(), "local"
    from torch._C._autograd import DeviceType
    from torch._C._distributed_c10d import _SymmetricMemory

    try:
        so = _symmetric_output(M, N, out_dtype, dev, group, lib)
    except RuntimeError:
        if not allow_unfused:
            raise
        out = local_product()
        dist.all_reduce(out, group=group)
        return out, "unfused-nccl"
    has_mc = bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, dev.index)) and bool(so.hdl.multicast_ptr)
    if method == "auto":
        if out_dtype == torch.bfloat16:
            method = "peer" if (world == 2 or not has_mc) else "two-phase"
        elif has_mc and M * N * 4 <= ONE_SHOT_MAX_BYTES:
            method = "one-shot"
        else:
            method = "peer" if (world == 2 or not has_mc) else "two-phase"
    if method in ("one-shot", "two-phase") and not has_mc:
        raise RuntimeError(f"no NVSwitch multicast for this group: method {method!r} is unavailable (use 'peer')")
    if method == "one-shot":
        so.out.zero_()
        so.hdl.barrier(channel=0, timeout_ms=_BARRIER_TIMEOUT_MS)  # every copy is zero before anyone adds
        _lib.check(lib.kdn_tp_out_proj(y.data_ptr(), w.data_ptr(), None, _lib.KDN_DTYPE_F32, so.multicast(), M, N, K,
                                       stream), "kdn_tp_out_proj")
    else:
        so.calls += 1
        target = (so.calls * world) & 0xFFFFFFFF
        if method == "two-phase":
            rc = lib.kdn_tp_out_proj_allreduce(y.data_ptr(), w.data_ptr(), so.out.data_ptr(), so.multicast(),
                                               _lib.dtype_code(so.out), so.counters.data_ptr(),
                                               so.multicast(so.ctr_off), target, rank, world, M, N, K, stream)
        else:
            outs = (ctypes.c_void_p * world)(*so.peer_ptrs(0))
            ctrs = (ctypes.c_void_p * world)(*so.peer_ptrs(so.ctr_off))
            rc = lib.kdn_tp_out_proj_allreduce_peer(y.data_ptr(), w.data_ptr(), outs, _lib.dtype_code(so.out), ctrs,
                                                    target, rank, world, M, N, K, stream)
        _lib.check(rc, "kdn_tp_out_proj_allreduce")
    so.hdl.barrier(channel=0, timeout_ms=_BARRIER_TIMEOUT_MS)  # every rank's tiles are in every copy
    return so.out, "fused-" + method


def release_symmetric_buffers() -> None:
    """Drop the cached symmetric output buffers (call before destroying the process group)."""
    _SYMM.clear()
