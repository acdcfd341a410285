"""Ragged (varlen) prefill over a slot-mapped state pool -- the serving-side prefill.

The reference's ragged engine packs requests into one token dimension with
``cu_seqlens`` metadata and then runs each request separately
(serving/vllm_ragged_batching.py:41-103); its state pool (serving/hybrid_memory_pool.cpp)
keeps one recurrent state per stream.  Here:

    ragged_prefill(query, key, value, beta, decay, cu_seqlens, recurrent_states,
                   slot_mapping, output, fwht_proj=None, chunk_size=64, mode=None,
                   initial_state_mask=None, head_major_inputs=False)

* ``query``/``key`` [total_tokens, H, d_k], ``value``/``output`` [total_tokens, H, d_v],
  ``beta``/``decay`` [total_tokens, H] (``decay`` may be None: 1), packed back to back;
  ``cu_seqlens`` [num_seqs + 1] (nondecreasing from 0 to total_tokens).
* ``recurrent_states`` [num_slots, H, d_v, D] float32 is the pool: sequence i starts from
  ``recurrent_states[slot_mapping[i]]`` and its final state is written back there, in
  place.  ``initial_state_mask[i] = False`` starts sequence i from zeros instead (a new
  request whose slot holds a stale state).  Slots must be distinct.
* ``output`` is written in place; everything runs on the current CUDA stream.
* ``head_major_inputs=True``: query/key/value/beta/decay (same shapes) already hold the
  per-sequence head-major layout below (as ``kdn_mixer_inputs`` writes it given
  ``cu_seqlens``), so their transposes are skipped; ``output`` stays packed.

The packed tensors are moved to per-sequence head-major blocks ([H, T_i, .], no padding)
by ``kdn_ragged_transpose``.  In bf16 mode a batch with at least as many (sequence, head)
scans as SMs then runs as ONE varlen launch (``kdn_chunked_prefill_varlen``: one CTA per
scan on the tensor-core path, longest first).  Otherwise each sequence runs the exact chunked
prefill of ``fused_chunked_deltanet_forward`` (so the arithmetic, paths and tolerances are those
of that op), several sequences in one call when they are adjacent, of equal length, and map to
consecutive slots.  ``fork_recurrent_state`` copies a slot for a forked request.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _lib
from ..kernels.fused_kernel_deltanet import fused_chunked_deltanet_forward
from ..kernels.fwht import FastWalshHadamardProjection
from .vllm_kernel_deltanet_op import default_projection


def _index_code(t: torch.Tensor) -> int:
    if t.dtype == torch.int64:
        return _lib.KDN_INDEX_I64
    if t.dtype == torch.int32:
        return _lib.KDN_INDEX_I32
    raise RuntimeError(f"cu_seqlens must be int32 or int64, got {t.dtype}")


def _to_head_major(lib, src: torch.Tensor, cu_dev: torch.Tensor, num_seqs: int, H: int, dev) -> torch.Tensor:
    total = src.shape[0]
    dst = torch.empty_like(src)
    row_bytes = (src[0, 0].numel() if src.dim() > 2 else 1) * src.element_size()
    rc = lib.kdn_ragged_transpose(src.data_ptr(), dst.data_ptr(), cu_dev.data_ptr(), _index_code(cu_dev), num_seqs,
                                  total, H, row_bytes, 1, _lib.stream_handle(dev))
    _lib.check(rc, "kdn_ragged_transpose")
    return dst


def _varlen_prefill(lib, qh, kh, vh, bh, dh, yh, lens, starts, sl, mask, pool, proj, H, dv, total, dev) -> bool:
    """All (sequence, head) scans of the batch in one launch (kdn_chunked_prefill_varlen: one CTA per
    scan on the tensor-core path), longest scans first; states gathered from and scattered back to the
    pool.  Used when the batch has more than one non-empty sequence and at least as many scans as SMs
    (fewer scans run better through the per-sequence path, which spreads a sequence over the GPU).
    Returns False when it does not apply."""
    live = [i for i, n in enumerate(lens) if n > 0]
    if len(live) < 2 or len(live) * H < torch.cuda.get_device_properties(dev).multi_processor_count:
        return False
    order = sorted(live, key=lambda i: -lens[i])
    offs = [starts[i] * H + h * lens[i] for i in order for h in range(H)]
    lns = [lens[i] for i in order for h in range(H)]
    rows = [sl[i] * H + h for i in order for h in range(H)]
    N = len(offs)
    view = pool.view(pool.shape[0] * H, dv, -1)
    rows_dev = torch.tensor(rows, device=dev, dtype=torch.int64)
    fresh = [mask is not None and not bool(mask[i]) for i in order]
    S0 = None
    if not all(fresh):
        S0 = view.index_select(0, rows_dev)
        if any(fresh):
            keep = torch.tensor([0.0 if f else 1.0 for f in fresh for _ in range(H)], device=dev)
            S0.mul_(keep[:, None, None])
    S_out = torch.empty(N, dv, view.shape[-1], device=dev, dtype=torch.float32)
    offs_dev = torch.tensor(offs, device=dev, dtype=torch.int64)
    lns_dev = torch.tensor(lns, device=dev, dtype=torch.int64)
    p, _phase = proj.kdn_projection(dev)
    rc = lib.kdn_chunked_prefill_varlen(
        qh.data_ptr(), kh.data_ptr(), vh.data_ptr(), _lib.dtype_code(qh), bh.data_ptr(), _lib.ptr(dh),
        _lib.dtype_code(bh), _lib.ptr(S0), yh.data_ptr(), _lib.dtype_code(yh), S_out.data_ptr(), offs_dev.data_ptr(),
        lns_dev.data_ptr(), N, total * H, dv, 64, p, _lib.stream_handle(dev))
    if rc == 2:  # KDN_ERR_UNSUPPORTED (e.g. a projection whose constants the tensor-core lift cannot hold)
        return False
    _lib.check(rc, "kdn_chunked_prefill_varlen")
    view.index_copy_(0, rows_dev, S_out)
    for i, n in enumerate(lens):  # empty sequences: a fresh one leaves a zero state
        if n == 0 and mask is not None and not bool(mask[i]):
            pool[sl[i]].zero_()
    return True


def ragged_prefill(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, beta: torch.Tensor,
                   decay: Optional[torch.Tensor], cu_seqlens: torch.Tensor, recurrent_states: torch.Tensor,
                   slot_mapping: torch.Tensor, output: torch.Tensor,
                   fwht_proj: Optional[FastWalshHadamardProjection] = None, chunk_size: int = 64,
                   mode: Optional[str] = None, initial_state_mask: Optional[torch.Tensor] = None,
                   head_major_inputs: bool = False) -> torch.Tensor:
    # ---------------------------------------------------------------- host-side checks
    if query.dim() != 3 or key.shape != query.shape:
        raise RuntimeError(f"query/key must be [total_tokens, H, d_k]; got {tuple(query.shape)}, {tuple(key.shape)}")
    total, H, d_k = query.shape
    if value.dim() != 3 or value.shape[:2] != (total, H):
        raise RuntimeError(f"value must be [total_tokens, H, d_v]; got {tuple(value.shape)}")
    dv = value.shape[2]
    if output.shape != value.shape:
        raise RuntimeError(f"output must be {tuple(value.shape)}; got {tuple(output.shape)}")
    if beta.shape != (total, H) or (decay is not None and decay.shape != (total, H)):
        raise RuntimeError("beta/decay must be [total_tokens, H]")
    cu = cu_seqlens.detach().to("cpu", torch.int64)
    if cu.dim() != 1 or cu.numel() < 2 or int(cu[0]) != 0 or int(cu[-1]) != total or bool((cu[1:] < cu[:-1]).any()):
        raise RuntimeError("cu_seqlens must be nondecreasing from 0 to total_tokens")
    num_seqs = cu.numel() - 1
    slots = slot_mapping.detach().to("cpu", torch.int64)
    if slots.shape != (num_seqs,):
        raise RuntimeError(f"slot_mapping must be [num_seqs] = [{num_seqs}]")
    if recurrent_states.dim() != 4 or recurrent_states.shape[1:3] != (H, dv):
        raise RuntimeError(f"recurrent_states must be [num_slots, H={H}, d_v={dv}, D]")
    num_slots = recurrent_states.shape[0]
    if num_seqs and (int(slots.min()) < 0 or int(slots.max()) >= num_slots):
        raise RuntimeError(f"slot_mapping out of range [0, {num_slots})")
    if torch.unique(slots).numel() != num_seqs:
        raise RuntimeError("slot_mapping must not map two sequences to one slot")
    mask = None
    if initial_state_mask is not None:
        mask = initial_state_mask.detach().to("cpu", torch.bool)
        if mask.shape != (num_seqs,):
            raise RuntimeError(f"initial_state_mask must be [num_seqs] = [{num_seqs}]")
    if recurrent_states.dtype != torch.float32 or not recurrent_states.is_contiguous():
        raise RuntimeError("recurrent_states must be a contiguous float32 pool")
    for t in (query, key, value, beta, decay, recurrent_states, output):
        if t is not None and not t.is_cuda:
            raise RuntimeError("kdn_b200 runs on CUDA tensors only (no CPU fallback)")
    dev = query.device
    proj = fwht_proj if fwht_proj is not None else default_projection(d_k, recurrent_states.shape[3])
    if proj.D != recurrent_states.shape[3] or proj.d_k != d_k:
        raise RuntimeError("projection sizes do not match the state pool / inputs")
    if total == 0:
        return output

    # ---------------------------------------------------------------- packed -> head-major
    lib = _lib.load()
    cu_dev = cu.to(dev)
    in_dtype = query.dtype if query.dtype in (torch.float32, torch.bfloat16) else torch.float32
    gate_dtype = beta.dtype if beta.dtype in (torch.float32, torch.bfloat16) else torch.float32
    if head_major_inputs:  # already laid out per sequence and head (kdn_mixer_inputs with cu_seqlens)
        qh, kh, vh = (t.to(in_dtype).contiguous() for t in (query, key, value))
        bh = beta.to(gate_dtype).contiguous()
        dh = decay.to(gate_dtype).contiguous() if decay is not None else None
    else:
        qh = _to_head_major(lib, query.to(in_dtype).contiguous(), cu_dev, num_seqs, H, dev)
        kh = _to_head_major(lib, key.to(in_dtype).contiguous(), cu_dev, num_seqs, H, dev)
        vh = _to_head_major(lib, value.to(in_dtype).contiguous(), cu_dev, num_seqs, H, dev)
        bh = _to_head_major(lib, beta.to(gate_dtype).contiguous(), cu_dev, num_seqs, H, dev)
        dh = (_to_head_major(lib, decay.to(gate_dtype).contiguous(), cu_dev, num_seqs, H, dev)
              if decay is not None else None)
    yh = torch.empty(total * H * dv, device=dev, dtype=output.dtype if output.dtype in (torch.float32, torch.bfloat16)
                     else in_dtype)

    lens = (cu[1:] - cu[:-1]).tolist()
    starts = cu[:-1].tolist()
    sl = slots.tolist()
    run_mode = mode or ("bf16" if in_dtype == torch.bfloat16 else "fp32")
    batched = (run_mode == "bf16" and d_k == 64 and dv == 64 and proj.D == 512 and chunk_size == 64
               and _varlen_prefill(lib, qh, kh, vh, bh, dh, yh, lens, starts, sl, mask, recurrent_states, proj, H,
                                   dv, total, dev))

    # ---------------------------------------------------------------- one prefill per run of sequences
    i = num_seqs if batched else 0
    while i < num_seqs:
        j = i + 1  # extend the run: equal length, next slot, same start rule
        while (j < num_seqs and lens[j] == lens[i] and sl[j] == sl[j - 1] + 1
               and (mask is None or bool(mask[j]) == bool(mask[i]))):
            j += 1
        g, T = j - i, lens[i]
        pool = recurrent_states[sl[i]:sl[i] + g].view(g * H, dv, -1)
        fresh = mask is not None and not bool(mask[i])
        if T == 0:
            if fresh:
                pool.zero_()
        else:
            t0 = starts[i] * H
            n = g * H * T
            view = lambda x, w: x[t0 * w:(t0 + n) * w].view(g * H, T, w) if w > 1 else x[t0:t0 + n].view(g * H, T)
            fused_chunked_deltanet_forward(view(qh.view(-1), d_k), view(kh.view(-1), d_k), view(vh.view(-1), dv),
                                           view(bh.view(-1), 1), view(dh.view(-1), 1) if dh is not None else None,
                                           proj, chunk_size, None if fresh else pool, mode=mode,
                                           out=yh[t0 * dv:(t0 + n) * dv].view(g * H, T, dv), final_state=pool)
        i = j

    # ---------------------------------------------------------------- head-major -> packed output
    out = output if output.dtype == yh.dtype and output.is_contiguous() else torch.empty_like(output, dtype=yh.dtype)
    rc = lib.kdn_ragged_transpose(yh.data_ptr(), out.data_ptr(), cu_dev.data_ptr(), _index_code(cu_dev), num_seqs,
                                  total, H, dv * yh.element_size(), 0, _lib.stream_handle(dev))
    _lib.check(rc, "kdn_ragged_transpose")
    if out is not output:
        output.copy_(out)
    return output
