"""Exact gated delta-rule chunked prefill -- drop-in for kernels/fused_kernel_deltanet.py.

``fused_chunked_deltanet_forward(q, k, v, beta, decay, fwht_proj, chunk_size,
initial_state) -> (Y, S)`` keeps the reference signature and meaning
(kernels/fused_kernel_deltanet.py:31-40):

    S_t = decay_t S_{t-1} (I - beta_t phi(k_t) phi(k_t)^T) + beta_t v_t phi(k_t)^T
    y_t = S_{t-1} phi(q_t)

with q, k [B, T, d_k], v [B, T, d_v], beta/decay [B, T], state [B, d_v, D]
(heads flattened into B by the caller, as in pipeline/transmute.py:75-79).
Y is returned in q's dtype; the state is always returned in float32 (the
reference keeps it in the input dtype -- fp32 state is this build's contract).

Arithmetic modes: ``"fp32"`` (fp32: CUDA cores and split-tf32 tensor-core products, 1e-4 of the
fp32 reference) and ``"bf16"`` (bf16
tensor-core products with fp32 accumulation and fp32 state); default: "bf16"
for bfloat16 inputs, "fp32" otherwise.  The work runs in libkdn on the
tensors' CUDA device and current stream; there is no CPU path.  Host
(CPU) tensors are accepted with ``device="cuda"``: the sequence is then streamed
through that device in segments of ``segment_tokens`` (copies in and out overlap
the kernels) and the results come back as host tensors, complete on return.
Gradients: when any of q, k, v, beta, decay, initial_state requires grad (and grad mode
is on), the call goes through an autograd Function whose backward is the libkdn backward
(``kdn_chunked_prefill_backward``: exact fp32, forward recomputed with chunk checkpoints),
for dY and d(final state) alike; the reference gets the same gradients by recompute +
autograd (:158-179).  ``chunked_deltanet_backward`` exposes that backward directly.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from .. import _lib
from .fwht import FastWalshHadamardProjection

_MODES = {"fp32": _lib.KDN_MODE_F32, "bf16": _lib.KDN_MODE_BF16}


def _check_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("kdn_b200 runs on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def fused_chunked_deltanet_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    beta: torch.Tensor,
    decay: Optional[torch.Tensor],
    fwht_proj: FastWalshHadamardProjection,
    chunk_size: int = 64,
    initial_state: Optional[torch.Tensor] = None,
    *,
    mode: Optional[str] = None,
    workspace: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    final_state: Optional[torch.Tensor] = None,
    device=None,
    segment_tokens: int = 8192,
) -> Tuple[torch.Tensor, torch.Tensor]:
    needs_grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (q, k, v, beta, decay, initial_state))
    if needs_grad:
        if out is not None or final_state is not None or not q.is_cuda:
            raise RuntimeError("inputs that require grad take neither out=/final_state= buffers nor host tensors")
        return _PrefillWithGrad.apply(q, k, v, beta, decay, initial_state, fwht_proj, chunk_size, mode)
    return _forward_impl(q, k, v, beta, decay, fwht_proj, chunk_size, initial_state, mode=mode, workspace=workspace,
                         out=out, final_state=final_state, device=device, segment_tokens=segment_tokens)


def _forward_impl(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    beta: torch.Tensor,
    decay: Optional[torch.Tensor],
    fwht_proj: FastWalshHadamardProjection,
    chunk_size: int = 64,
    initial_state: Optional[torch.Tensor] = None,
    *,
    mode: Optional[str] = None,
    workspace: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    final_state: Optional[torch.Tensor] = None,
    device=None,
    segment_tokens: int = 8192,
) -> Tuple[torch.Tensor, torch.Tensor]:
    if not q.is_cuda:
        if device is None:
            raise RuntimeError("kdn_b200 runs on CUDA tensors only (no CPU fallback); pass device='cuda' to stream "
                               "host tensors through the GPU")
        return _streamed_forward(q, k, v, beta, decay, fwht_proj, chunk_size, initial_state, mode,
                                 torch.device(device), out, final_state, segment_tokens)
    dev = _check_cuda(q, k, v, beta, decay, initial_state)
    if q.dim() != 3 or k.shape != q.shape or v.dim() != 3 or v.shape[:2] != q.shape[:2]:
        raise RuntimeError(f"expected q,k [B,T,d_k] and v [B,T,d_v]; got {tuple(q.shape)}, {tuple(k.shape)}, "
                           f"{tuple(v.shape)}")
    B, T, d_k = q.shape
    dv = v.shape[-1]
    D = fwht_proj.D
    if d_k != fwht_proj.d_k:
        raise RuntimeError(f"d_k {d_k} != projection d_k {fwht_proj.d_k}")
    if beta.shape != (B, T) or (decay is not None and decay.shape != (B, T)):
        raise RuntimeError("beta/decay must be [B, T]")
    if mode is None:
        mode = "bf16" if q.dtype == torch.bfloat16 else "fp32"
    if mode not in _MODES:
        raise RuntimeError(f"mode must be one of {sorted(_MODES)}")
    in_dtype = q.dtype if q.dtype in (torch.float32, torch.bfloat16) else torch.float32
    q = q.to(in_dtype).contiguous()
    k = k.to(in_dtype).contiguous()
    v = v.to(in_dtype).contiguous()
    gate_dtype = beta.dtype if beta.dtype in (torch.float32, torch.bfloat16) else torch.float32
    beta = beta.to(gate_dtype).contiguous()
    if decay is not None:
        decay = decay.to(gate_dtype).contiguous()
    S0 = None
    if initial_state is not None:
        if initial_state.shape != (B, dv, D):
            raise RuntimeError(f"initial_state must be [B, d_v, D] = {(B, dv, D)}")
        S0 = initial_state.to(torch.float32).contiguous()

    y = out if out is not None else torch.empty(B, T, dv, device=dev, dtype=in_dtype)
    S = final_state if final_state is not None else torch.empty(B, dv, D, device=dev, dtype=torch.float32)
    lib = _lib.load()
    proj, _phase = fwht_proj.kdn_projection(dev)
    mcode = _MODES[mode]
    ws_bytes = int(lib.kdn_chunked_prefill_workspace_size(B, T, dv, chunk_size, proj, mcode))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    rc = lib.kdn_chunked_prefill(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.dtype_code(q),
        beta.data_ptr(), _lib.ptr(decay), _lib.dtype_code(beta),
        _lib.ptr(S0), y.data_ptr(), _lib.dtype_code(y), S.data_ptr(),
        B, T, dv, chunk_size, proj, mcode, workspace.data_ptr(), ws_bytes, _lib.stream_handle(dev))
    _lib.check(rc, "kdn_chunked_prefill")
    return y, S


def _copy_rows(lib, dst, src, stream):
    """dst[b, :n] = src[b, :n] for every b (same dtype; rows contiguous inside, pitched between)."""
    rows, n = src.shape[0], src.shape[1]
    esz = src.element_size()
    width = n * (src[0, 0].numel()) * esz
    rc = lib.kdn_copy_rows(dst.data_ptr(), dst.stride(0) * esz, src.data_ptr(), src.stride(0) * esz, width, rows,
                           stream.cuda_stream)
    _lib.check(rc, "kdn_copy_rows")


def _segment_plan(T: int, seg: int, chunk: int):
    """Token ranges [(t0, t1)] of the streamed segments, whole chunks except the ragged end of the
    sequence.  The middle segments are `seg` tokens long (few calls, small per-call overhead); the
    sequence starts and ends with ramps of seg/8, seg/4 and seg/2 tokens, because the copy-in of the
    first segment and the compute and copy-out of the last one overlap nothing."""
    seg_c = max(1, seg // chunk)
    n_c = (T + chunk - 1) // chunk
    ramp = sorted({r for r in (seg_c // 8, seg_c // 4, seg_c // 2) if 1 <= r < seg_c})
    if n_c <= 2 * sum(ramp) + seg_c:
        sizes = [seg_c] * (n_c // seg_c) + ([n_c % seg_c] if n_c % seg_c else [])
    else:
        mid = n_c - 2 * sum(ramp)
        sizes = ramp + [seg_c] * (mid // seg_c) + ([mid % seg_c] if mid % seg_c else []) + ramp[::-1]
    plan, c0 = [], 0
    for sz in sizes:
        plan.append((c0 * chunk, min(T, (c0 + sz) * chunk)))
        c0 += sz
    return plan


def _streamed_forward(q, k, v, beta, decay, fwht_proj, chunk_size, initial_state, mode, dev, out, final_state,
                      segment_tokens):
    """Host tensors in, host tensors out, the work on `dev`: the sequence is cut into segments of whole
    chunks (`_segment_plan`); while segment i runs, the inputs of segment i+1 are copied in and the
    outputs of segment i-1 are copied out (two copy streams, three device segment buffers).  The fp32
    state is carried from segment to segment on the device, so the result equals one call over the
    whole sequence (the chunks and their arithmetic are the same)."""
    if dev.type != "cuda":
        raise RuntimeError(f"device must be a CUDA device, got {dev}")
    for t in (k, v, beta, decay, initial_state, out, final_state):
        if t is not None and t.is_cuda:
            raise RuntimeError("stream from the host: every tensor argument must be a host tensor")
    if q.dim() != 3 or k.shape != q.shape or v.dim() != 3 or v.shape[:2] != q.shape[:2]:
        raise RuntimeError(f"expected q,k [B,T,d_k] and v [B,T,d_v]; got {tuple(q.shape)}, {tuple(k.shape)}, "
                           f"{tuple(v.shape)}")
    B, T, d_k = q.shape
    dv = v.shape[-1]
    D = fwht_proj.D
    if beta.shape != (B, T) or (decay is not None and decay.shape != (B, T)):
        raise RuntimeError("beta/decay must be [B, T]")
    in_dtype = q.dtype if q.dtype in (torch.float32, torch.bfloat16) else torch.float32
    gate_dtype = beta.dtype if beta.dtype in (torch.float32, torch.bfloat16) else torch.float32
    src = [t.to(dt).contiguous() for t, dt in ((q, in_dtype), (k, in_dtype), (v, in_dtype))]
    gates = [beta.to(gate_dtype).contiguous()] + ([decay.to(gate_dtype).contiguous()] if decay is not None else [])
    y_host = out if out is not None else torch.empty(B, T, dv, dtype=in_dtype, pin_memory=True)
    if y_host.shape != (B, T, dv) or y_host.dtype != in_dtype or not y_host.is_contiguous():
        raise RuntimeError(f"out must be a contiguous host tensor [B, T, d_v] of {in_dtype}")
    S_host = final_state if final_state is not None else torch.empty(B, dv, D, dtype=torch.float32, pin_memory=True)
    if S_host.shape != (B, dv, D) or S_host.dtype != torch.float32 or not S_host.is_contiguous():
        raise RuntimeError("final_state must be a contiguous host float32 tensor [B, d_v, D]")
    seg = max(chunk_size, (int(segment_tokens) // chunk_size) * chunk_size)
    plan = _segment_plan(T, seg, chunk_size)
    seg = max([t1 - t0 for t0, t1 in plan], default=chunk_size)  # the longest segment sizes the buffers
    proj = fwht_proj  # its device constants are built per device on demand
    compute = torch.cuda.current_stream(dev)
    copy_in = torch.cuda.Stream(dev)
    copy_out = torch.cuda.Stream(dev)
    # a segment of n tokens views the first B*n rows of its flat buffers as contiguous [B, n, ...] tensors
    view = lambda flat, n, *tail: flat[:B * n * (tail[0] if tail else 1)].view(B, n, *tail)
    with torch.cuda.device(dev):
        nb = 3  # three segment buffers: a short segment's copy-in never waits for the copy-out two back
        dsrc = [[torch.empty(B * seg * t.shape[-1], dtype=t.dtype, device=dev) for t in src] for _ in range(nb)]
        dgate = [[torch.empty(B * seg, dtype=g.dtype, device=dev) for g in gates] for _ in range(nb)]
        dy = [torch.empty(B * seg * dv, dtype=in_dtype, device=dev) for _ in range(nb)]
        dS = [torch.empty(B, dv, D, dtype=torch.float32, device=dev) for _ in range(2)]
        if initial_state is not None:
            if initial_state.shape != (B, dv, D):
                raise RuntimeError(f"initial_state must be [B, d_v, D] = {(B, dv, D)}")
            dS[1].copy_(initial_state.to(torch.float32), non_blocking=False)
        lib = _lib.load()
        pstruct, _phase = proj.kdn_projection(dev)
        mcode = _MODES[mode if mode is not None else ("bf16" if in_dtype == torch.bfloat16 else "fp32")]
        ws_bytes = int(lib.kdn_chunked_prefill_workspace_size(B, seg, dv, chunk_size, pstruct, mcode))
        ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
        freed = [torch.cuda.Event() for _ in range(nb)]   # segment buffer i % nb may be refilled
        loaded = [torch.cuda.Event() for _ in range(nb)]
        done = [torch.cuda.Event() for _ in range(nb)]
        nseg = len(plan)
        S_prev = dS[1] if initial_state is not None else None
        for i, (t0, t1) in enumerate(plan):
            n = t1 - t0
            b = i % nb
            qq, kk, vv = (view(x, n, t.shape[-1]) for x, t in zip(dsrc[b], src))
            gg = [view(x, n) for x in dgate[b]]
            yy = view(dy[b], n, dv)
            with torch.cuda.stream(copy_in):
                if i >= nb:
                    copy_in.wait_event(freed[b])
                for hs, ds in zip(src + gates, [qq, kk, vv] + gg):  # one strided copy per tensor
                    _copy_rows(lib, ds, hs[:, t0:t1], copy_in)
                loaded[b].record(copy_in)
            compute.wait_event(loaded[b])
            S_next = dS[i % 2]
            dd = gg[1] if decay is not None else None
            fused_chunked_deltanet_forward(qq, kk, vv, gg[0], dd, proj, chunk_size, S_prev, mode=mode,
                                           workspace=ws, out=yy, final_state=S_next)
            done[b].record(compute)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(done[b])
                _copy_rows(lib, y_host[:, t0:t1], yy[:, :n], copy_out)
                if i == nseg - 1:
                    S_host.copy_(S_next, non_blocking=True)
                freed[b].record(copy_out)
            yy.record_stream(copy_out)
            S_prev = S_next
        if nseg == 0:  # T == 0: the state passes through
            S_host.copy_(initial_state.to(torch.float32) if initial_state is not None else torch.zeros_like(S_host))
        compute.wait_stream(copy_out)
        compute.synchronize()  # host results are complete when the call returns
    return y_host, S_host


def chunked_deltanet_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                              decay: Optional[torch.Tensor], dY: torch.Tensor,
                              fwht_proj: FastWalshHadamardProjection, chunk_size: int = 64,
                              initial_state: Optional[torch.Tensor] = None,
                              d_final_state: Optional[torch.Tensor] = None) -> dict:
    """Gradients of the chunked prefill (libkdn ``kdn_chunked_prefill_backward``, exact fp32).

    Same shapes as the forward; dY [B, T, d_v] is dL/dY and d_final_state [B, d_v, D] (or None)
    dL/d(final state).  Returns fp32 tensors {"dq", "dk", "dv", "dbeta", "ddecay" (None without
    decay), "d_initial_state"} -- the gradients the reference's recompute + autograd gives
    (kernels/fused_kernel_deltanet.py:167-179), plus the initial state's."""
    dev = _check_cuda(q, k, v, beta, decay, dY, initial_state, d_final_state)
    B, T, d_k = q.shape
    dv = v.shape[-1]
    D = fwht_proj.D
    if k.shape != q.shape or v.shape[:2] != (B, T) or dY.shape != v.shape or beta.shape != (B, T):
        raise RuntimeError("shape mismatch between q, k, v, beta and dY")
    in_dtype = q.dtype if q.dtype in (torch.float32, torch.bfloat16) else torch.float32
    gate_dtype = beta.dtype if beta.dtype in (torch.float32, torch.bfloat16) else torch.float32
    qc, kc, vc = (t.detach().to(in_dtype).contiguous() for t in (q, k, v))
    bc = beta.detach().to(gate_dtype).contiguous()
    dc = None if decay is None else decay.detach().to(gate_dtype).contiguous()
    yc = dY.detach().to(torch.float32 if dY.dtype not in (torch.float32, torch.bfloat16) else dY.dtype).contiguous()
    S0 = None if initial_state is None else initial_state.detach().to(torch.float32).contiguous()
    dSf = None if d_final_state is None else d_final_state.detach().to(torch.float32).contiguous()
    f32 = dict(device=dev, dtype=torch.float32)
    dq, dk = torch.empty(B, T, d_k, **f32), torch.empty(B, T, d_k, **f32)
    dvv = torch.empty(B, T, dv, **f32)
    db = torch.empty(B, T, **f32)
    dd = torch.empty(B, T, **f32) if dc is not None else None
    dS0 = torch.empty(B, dv, D, **f32)
    lib = _lib.load()
    proj, _phase = fwht_proj.kdn_projection(dev)
    ws_bytes = int(lib.kdn_chunked_prefill_backward_workspace_size(B, T, dv, chunk_size, proj))
    ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
    rc = lib.kdn_chunked_prefill_backward(
        qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), _lib.dtype_code(qc), bc.data_ptr(), _lib.ptr(dc),
        _lib.dtype_code(bc), _lib.ptr(S0), yc.data_ptr(), _lib.dtype_code(yc), _lib.ptr(dSf), dq.data_ptr(),
        dk.data_ptr(), dvv.data_ptr(), db.data_ptr(), _lib.ptr(dd), dS0.data_ptr(), B, T, dv, chunk_size, proj,
        ws.data_ptr(), ws_bytes, _lib.stream_handle(dev))
    _lib.check(rc, "kdn_chunked_prefill_backward")
    return {"dq": dq, "dk": dk, "dv": dvv, "dbeta": db, "ddecay": dd, "d_initial_state": dS0}


def _grad_as(g: Optional[torch.Tensor], like: Optional[torch.Tensor]):
    if g is None or like is None or not like.requires_grad:
        return None
    return g.to(like.dtype)


class _PrefillWithGrad(torch.autograd.Function):
    """(Y, final state) with the libkdn backward for both outputs."""

    @staticmethod
    def forward(ctx, q, k, v, beta, decay, initial_state, fwht_proj, chunk_size, mode):
        Y, S = _forward_impl(q, k, v, beta, decay, fwht_proj, chunk_size, initial_state, mode=mode)
        ctx.save_for_backward(q, k, v, beta, decay, initial_state)
        ctx.fwht_proj, ctx.chunk_size = fwht_proj, chunk_size
        return Y, S

    @staticmethod
    def backward(ctx, dY, dS):
        q, k, v, beta, decay, S0 = ctx.saved_tensors
        if dY is None:
            dY = torch.zeros(v.shape, device=v.device, dtype=torch.float32)
        g = chunked_deltanet_backward(q, k, v, beta, decay, dY, ctx.fwht_proj, ctx.chunk_size, S0, dS)
        return (_grad_as(g["dq"], q), _grad_as(g["dk"], k), _grad_as(g["dv"], v), _grad_as(g["dbeta"], beta),
                _grad_as(g["ddecay"], decay), _grad_as(g["d_initial_state"], S0), None, None, None)


class FusedKernelDeltaNetFunction(torch.autograd.Function):
    """Autograd Function of the reference (kernels/fused_kernel_deltanet.py:158-179): Y only.
    Its backward is the libkdn backward rather than recompute + autograd (same gradients)."""

    @staticmethod
    def forward(ctx, q, k, v, beta, decay, fwht_proj, chunk_size=64):
        Y, _ = _forward_impl(q, k, v, beta, decay, fwht_proj, chunk_size)
        ctx.save_for_backward(q, k, v, beta, decay)
        ctx.fwht_proj, ctx.chunk_size = fwht_proj, chunk_size
        return Y

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, beta, decay = ctx.saved_tensors
        g = chunked_deltanet_backward(q, k, v, beta, decay, grad_output, ctx.fwht_proj, ctx.chunk_size)
        return (g["dq"].to(q.dtype), g["dk"].to(k.dtype), g["dv"].to(v.dtype), g["dbeta"].to(beta.dtype),
                None if decay is None else g["ddecay"].to(decay.dtype), None, None)


class FusedKernelDeltaNet(nn.Module):
    """Module form (kernels/fused_kernel_deltanet.py:182-208)."""

    def __init__(self, d_model: int = 64, d_kernel: int = 512, chunk_size: int = 64, mode: Optional[str] = None):
        super().__init__()
        self.d_model = d_model
        self.d_kernel = d_kernel
        self.chunk_size = chunk_size
        self.mode = mode
        self.fwht_proj = FastWalshHadamardProjection(d_k=d_model, D=d_kernel)

    def forward(self, q, k, v, beta, decay, initial_state=None):
        return fused_chunked_deltanet_forward(q=q, k=k, v=v, beta=beta, decay=decay, fwht_proj=self.fwht_proj,
                                              chunk_size=self.chunk_size, initial_state=initial_state,
                                              mode=self.mode)
