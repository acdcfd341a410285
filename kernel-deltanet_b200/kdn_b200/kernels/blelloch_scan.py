"""Affine semigroup of block state maps -- drop-in for kernels/blelloch_scan.py.

The delta-rule state map of any block of tokens is affine in the entering
state, ``S_out = S_in A + B`` with ``A [D, D]`` and ``B [d_v, D]`` (batched over
the leading axis), and blocks compose as (kernels/blelloch_scan.py:42-56,
core/associative_algebra.py:45-60)

    (A1, B1) o (A2, B2) = (A1 A2, B1 A2 + B2).

Surfaces (same names, arguments and results as the reference):

    compose_transitions(T1, T2) -> (A, B)
    blelloch_prefix_scan(transitions, initial_state=None) -> [S_0, ..., S_{N_c-1}]
    sequential_prefix_scan(transitions, initial_state=None) -> same list

plus the producer of the maps for a block of tokens (the reference only
describes it, kernels/blelloch_scan.py:8-12):

    chunk_block_transition(k, v, beta, decay, fwht_proj, chunk_size) -> (A, B)

All arithmetic is fp32 on CUDA cores in libkdn (``kdn_affine_compose``,
``kdn_affine_prefix_states``, ``kdn_block_transition``); inputs of another
float dtype are computed in fp32 and returned in their own dtype.  Both scans
return the same states: the library walks the state chain (a d_v x D x D
product per block) rather than the reference's up/down-sweep tree of D x D
compositions, which gives the identical prefix states with D/d_v times fewer
FLOPs.  There is no CPU path.
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from .. import _lib
from .fwht import FastWalshHadamardProjection

Transition = Tuple[torch.Tensor, torch.Tensor]


def _cuda_f32(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{name}: kdn_b200 runs on CUDA tensors only (no CPU fallback)")
    if not t.is_floating_point():
        raise RuntimeError(f"{name}: floating-point tensor expected, got {t.dtype}")
    return t.to(torch.float32).contiguous()


def _pad16(n: int) -> int:
    return (n + 15) // 16 * 16


def _pad_to(t: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    r, c = t.shape[-2:]
    if r == rows and c == cols:
        return t
    return F.pad(t, (0, cols - c, 0, rows - r))


def compose_transitions(T1: Transition, T2: Transition) -> Transition:
    """(A1, B1) o (A2, B2) = (A1 @ A2, B1 @ A2 + B2); A [B, D, D], B [B, d_v, D].

    Same surface as kernels/blelloch_scan.py:42-56.  Dimensions that are not
    multiples of 16 are zero-padded for the kernel (exact) and sliced back.
    """
    A1, B1 = T1
    A2, B2 = T2
    if A1.dim() != 3 or A1.shape != A2.shape or A1.shape[-1] != A1.shape[-2]:
        raise RuntimeError(f"A1, A2 must be [B, D, D]; got {tuple(A1.shape)}, {tuple(A2.shape)}")
    batch, D, _ = A1.shape
    if B1.dim() != 3 or B1.shape != B2.shape or B1.shape[0] != batch or B1.shape[-1] != D:
        raise RuntimeError(f"B1, B2 must be [B, d_v, D]; got {tuple(B1.shape)}, {tuple(B2.shape)}")
    dv = B1.shape[1]
    out_dtype = torch.promote_types(A1.dtype, B1.dtype)
    dev = A1.device
    a1, b1, a2, b2 = (_cuda_f32(t, n) for t, n in ((A1, "A1"), (B1, "B1"), (A2, "A2"), (B2, "B2")))
    Dp, dvp = _pad16(D), _pad16(dv)
    a1, a2 = _pad_to(a1, Dp, Dp).contiguous(), _pad_to(a2, Dp, Dp).contiguous()
    b1, b2 = _pad_to(b1, dvp, Dp).contiguous(), _pad_to(b2, dvp, Dp).contiguous()
    A = torch.empty(batch, Dp, Dp, device=dev, dtype=torch.float32)
    B = torch.empty(batch, dvp, Dp, device=dev, dtype=torch.float32)
    lib = _lib.load()
    rc = lib.kdn_affine_compose(a1.data_ptr(), b1.data_ptr(), a2.data_ptr(), b2.data_ptr(), A.data_ptr(),
                                B.data_ptr(), batch, Dp, dvp, _lib.stream_handle(dev))
    _lib.check(rc, "kdn_affine_compose")
    return A[:, :D, :D].to(out_dtype), B[:, :dv, :D].to(out_dtype)


def prefix_states(A: torch.Tensor, B: torch.Tensor, initial_state: Optional[torch.Tensor] = None,
                  want_final: bool = False):
    """Stacked form: A [N_c, B, D, D], B [N_c, B, d_v, D] -> states [N_c, B, d_v, D]
    (states[c] = the state entering block c), and the state after the last block
    when ``want_final``.  fp32 in and out; D and d_v multiples of 16."""
    if A.dim() != 4 or B.dim() != 4 or A.shape[:2] != B.shape[:2] or A.shape[-1] != A.shape[-2] \
            or B.shape[-1] != A.shape[-1]:
        raise RuntimeError(f"expected A [N_c, B, D, D] and B [N_c, B, d_v, D]; got {tuple(A.shape)}, {tuple(B.shape)}")
    n_c, batch, D, _ = A.shape
    dv = B.shape[2]
    a = _cuda_f32(A, "A")
    b = _cuda_f32(B, "B")
    s0 = None
    if initial_state is not None:
        if initial_state.shape != (batch, dv, D):
            raise RuntimeError(f"initial_state must be [B, d_v, D] = {(batch, dv, D)}")
        s0 = _cuda_f32(initial_state, "initial_state")
    dev = A.device
    states = torch.empty(max(n_c, 1), batch, dv, D, device=dev, dtype=torch.float32)
    final = torch.empty(batch, dv, D, device=dev, dtype=torch.float32) if want_final else None
    lib = _lib.load()
    rc = lib.kdn_affine_prefix_states(a.data_ptr(), b.data_ptr(), _lib.ptr(s0), states.data_ptr(), _lib.ptr(final),
                                      n_c, batch, D, dv, _lib.stream_handle(dev))
    _lib.check(rc, "kdn_affine_prefix_states")
    states = states[:n_c]
    return (states, final) if want_final else states


def _stack(transitions: Sequence[Transition]):
    if len(transitions) == 0:
        raise RuntimeError("at least one transition is required")
    A = torch.stack([t[0] for t in transitions])
    B = torch.stack([t[1] for t in transitions])
    return A, B


def _scan(transitions: Sequence[Transition], initial_state: Optional[torch.Tensor]) -> List[torch.Tensor]:
    A, B = _stack(transitions)
    n_c, batch, D, _ = A.shape
    dv = B.shape[2]
    out_dtype = A.dtype
    Dp, dvp = _pad16(D), _pad16(dv)
    s0 = initial_state
    if Dp != D or dvp != dv:
        A = _pad_to(A.float(), Dp, Dp)
        B = _pad_to(B.float(), dvp, Dp)
        if s0 is not None:
            s0 = _pad_to(s0.float(), dvp, Dp)
    states = prefix_states(A, B, s0)
    return [s[:, :dv, :D].to(out_dtype) for s in states.unbind(0)]


def blelloch_prefix_scan(transitions: Sequence[Transition],
                         initial_state: Optional[torch.Tensor] = None) -> List[torch.Tensor]:
    """Prefix boundary states [S_0, ..., S_{N_c-1}] of N_c transitions
    (kernels/blelloch_scan.py:59-125): S_c = S_0 A_{0..c-1} + B_{0..c-1}."""
    return _scan(transitions, initial_state)


def sequential_prefix_scan(transitions: Sequence[Transition],
                           initial_state: Optional[torch.Tensor] = None) -> List[torch.Tensor]:
    """The reference's sequential scan (kernels/blelloch_scan.py:128-150); same result."""
    return _scan(transitions, initial_state)


def chunk_block_transition(k: torch.Tensor, v: Optional[torch.Tensor], beta: torch.Tensor,
                           decay: Optional[torch.Tensor], fwht_proj: FastWalshHadamardProjection,
                           chunk_size: int = 64, *, want_A: bool = True, workspace: Optional[torch.Tensor] = None
                           ) -> Transition:
    """Affine map (A [N, D, D], B [N, d_v, D]) of a block of tokens: for every
    entering state S_in, the chunked prefill over the block leaves S_in A + B.
    k [N, T, d_k], v [N, T, d_v] (None: B is not computed and returned as None),
    beta/decay [N, T] (decay None means 1).  Exact fp32.  ``want_A=False`` skips A."""
    dev = k.device
    if not k.is_cuda:
        raise RuntimeError("kdn_b200 runs on CUDA tensors only (no CPU fallback)")
    if k.dim() != 3:
        raise RuntimeError(f"k must be [N, T, d_k]; got {tuple(k.shape)}")
    N, T, d_k = k.shape
    if d_k != fwht_proj.d_k:
        raise RuntimeError(f"d_k {d_k} != projection d_k {fwht_proj.d_k}")
    D = fwht_proj.D
    in_dtype = k.dtype if k.dtype in (torch.float32, torch.bfloat16) else torch.float32
    k = k.to(in_dtype).contiguous()
    dv = 0
    if v is not None:
        if v.dim() != 3 or v.shape[:2] != (N, T):
            raise RuntimeError(f"v must be [N, T, d_v]; got {tuple(v.shape)}")
        dv = v.shape[-1]
        v = v.to(in_dtype).contiguous()
    if beta.shape != (N, T) or (decay is not None and decay.shape != (N, T)):
        raise RuntimeError("beta/decay must be [N, T]")
    gate_dtype = beta.dtype if beta.dtype in (torch.float32, torch.bfloat16) else torch.float32
    beta = beta.to(gate_dtype).contiguous()
    if decay is not None:
        decay = decay.to(gate_dtype).contiguous()
    A = torch.empty(N, D, D, device=dev, dtype=torch.float32) if want_A else None
    B = torch.empty(N, dv, D, device=dev, dtype=torch.float32) if v is not None else None
    lib = _lib.load()
    proj, _phase = fwht_proj.kdn_projection(dev)
    ws_bytes = int(lib.kdn_block_transition_workspace_size(N, T, chunk_size, proj))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    rc = lib.kdn_block_transition(k.data_ptr(), _lib.ptr(v), _lib.dtype_code(k), beta.data_ptr(), _lib.ptr(decay),
                                  _lib.dtype_code(beta), _lib.ptr(A), _lib.ptr(B), N, T, max(dv, 16), chunk_size,
                                  proj, workspace.data_ptr(), ws_bytes, _lib.stream_handle(dev))
    _lib.check(rc, "kdn_block_transition")
    return A, B
