"""Serving decode ops -- drop-in for serving/vllm_kernel_deltanet_op.cpp.

``hybrid_recurrent_forward(query, key, value, beta, decay, recurrent_states,
slot_mapping, output)`` keeps the reference op's argument list and in-place
contract (serving/vllm_kernel_deltanet_op.cpp:11-20): every tensor belongs to
the caller, ``recurrent_states`` [num_slots, H, d_v, D] and ``output``
[num_tokens, H, d_v] are written in place, nothing is allocated, and the work
is enqueued on the current CUDA stream.  The reference op's body is empty; the
semantics implemented are the module decode loop of
kernels/kernel_deltanet_fused.py:288-300 (read out before the update).
``readout="post"`` reproduces benchmarks/run_full_batch_decoding.py:43-54.
A negative slot marks a padding token (its output row is zeroed).

``fork_recurrent_state(recurrent_states, parent_slot, child_slot)`` copies one
slot onto another on the current stream (serving/vllm_kernel_deltanet_op.cpp:39-58).
Errors raise RuntimeError, like the reference's TORCH_CHECK.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _lib
from ..kernels.fwht import FastWalshHadamardProjection

_DEFAULT_PROJ: dict = {}


def default_projection(d_k: int = 64, D: int = 512, seed: int = 42) -> FastWalshHadamardProjection:
    key = (d_k, D, seed)
    if key not in _DEFAULT_PROJ:
        _DEFAULT_PROJ[key] = FastWalshHadamardProjection(d_k, D, seed)
    return _DEFAULT_PROJ[key]


def hybrid_recurrent_forward(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, beta: torch.Tensor,
                             decay: Optional[torch.Tensor], recurrent_states: torch.Tensor,
                             slot_mapping: torch.Tensor, output: torch.Tensor,
                             fwht_proj: Optional[FastWalshHadamardProjection] = None,
                             readout: str = "pre") -> None:
    for name, t in (("query", query), ("key", key), ("value", value), ("beta", beta),
                    ("recurrent_states", recurrent_states), ("slot_mapping", slot_mapping), ("output", output)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be on CUDA")
    if decay is not None and not decay.is_cuda:
        raise RuntimeError("decay must be on CUDA")
    Ntok, H, d_k = query.shape
    dv = value.shape[-1]
    S_slots, H2, dv2, D = recurrent_states.shape
    if key.shape != query.shape or value.shape != (Ntok, H, dv) or output.shape != (Ntok, H, dv):
        raise RuntimeError("query/key [N,H,d_k], value/output [N,H,d_v] shape mismatch")
    if (H2, dv2) != (H, dv):
        raise RuntimeError(f"recurrent_states [S,H,d_v,D] = {tuple(recurrent_states.shape)} does not match H={H}, d_v={dv}")
    if beta.shape != (Ntok, H) or (decay is not None and decay.shape != (Ntok, H)):
        raise RuntimeError("beta/decay must be [num_tokens, num_heads]")
    if slot_mapping.shape != (Ntok,) or slot_mapping.dtype not in (torch.int32, torch.int64):
        raise RuntimeError("slot_mapping must be int32/int64 [num_tokens]")
    for name, t in (("recurrent_states", recurrent_states), ("output", output), ("slot_mapping", slot_mapping)):
        if not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous (it is written or indexed in place)")
    proj_mod = fwht_proj if fwht_proj is not None else default_projection(d_k, D)
    if proj_mod.D != D or proj_mod.d_k != d_k:
        raise RuntimeError("projection shape does not match query / recurrent_states")
    dev = query.device
    q = query.contiguous()
    k = key.to(q.dtype).contiguous()
    v = value.to(q.dtype).contiguous()
    b = beta.contiguous()
    d = None if decay is None else decay.to(b.dtype).contiguous()
    lib = _lib.load()
    proj, _phase = proj_mod.kdn_projection(dev)
    idx = _lib.KDN_INDEX_I64 if slot_mapping.dtype == torch.int64 else _lib.KDN_INDEX_I32
    ro = {"pre": _lib.KDN_READOUT_PRE, "post": _lib.KDN_READOUT_POST}[readout]
    rc = lib.kdn_decode_step(q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.dtype_code(q), b.data_ptr(),
                             _lib.ptr(d), _lib.dtype_code(b), recurrent_states.data_ptr(),
                             _lib.dtype_code(recurrent_states), S_slots, slot_mapping.data_ptr(), idx,
                             output.data_ptr(), _lib.dtype_code(output), Ntok, H, dv, proj, ro,
                             _lib.stream_handle(dev))
    _lib.check(rc, "kdn_decode_step")


def fork_recurrent_state(recurrent_states: torch.Tensor, parent_slot: int, child_slot: int) -> None:
    if not recurrent_states.is_cuda:
        raise RuntimeError("State buffer must be CUDA tensor")
    if not recurrent_states.is_contiguous():
        raise RuntimeError("State buffer must be contiguous")
    lib = _lib.load()
    per_slot = recurrent_states[0].numel() * recurrent_states.element_size()
    rc = lib.kdn_fork_state(recurrent_states.data_ptr(), recurrent_states.shape[0], per_slot, int(parent_slot),
                            int(child_slot), _lib.stream_handle(recurrent_states.device))
    _lib.check(rc, "kdn_fork_state")


def device_error(stream_device=None) -> int:
    """Read and clear the device-side bounds-check word (synchronises the current stream)."""
    lib = _lib.load()
    import ctypes

    code = ctypes.c_int(0)
    dev = torch.device("cuda", torch.cuda.current_device()) if stream_device is None else torch.device(stream_device)
    _lib.check(lib.kdn_device_error(_lib.stream_handle(dev), ctypes.byref(code)), "kdn_device_error")
    return code.value
