"""ctypes binding of libkdn.so (the C ABI declared in include/kdn.h).

There is no fallback: if the library is missing or a call fails, a
RuntimeError is raised (the same convention as the reference's TORCH_CHECK,
serving/vllm_kernel_deltanet_op.cpp:21-22).
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("KDN_LIB", os.path.join(_HERE, "libkdn.so"))

KDN_OK = 0
KDN_DTYPE_F32 = 0
KDN_DTYPE_BF16 = 1
KDN_INDEX_I32 = 0
KDN_INDEX_I64 = 1
KDN_MODE_F32 = 0
KDN_MODE_BF16 = 1
KDN_READOUT_PRE = 0
KDN_READOUT_POST = 1
ABI_VERSION = 1

_ERR_NAMES = {1: "KDN_ERR_INVALID", 2: "KDN_ERR_UNSUPPORTED", 3: "KDN_ERR_CUDA", 4: "KDN_ERR_WORKSPACE",
              5: "KDN_ERR_DEVICE"}


class KdnProjection(ctypes.Structure):
    """Mirror of ``kdn_projection`` (include/kdn.h)."""

    _fields_ = [
        ("d_k", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("tau_inv", ctypes.c_float),
        ("amp", ctypes.c_float),
        ("sign_bits", (ctypes.c_uint64 * 3) * 8),
        ("phase", ctypes.c_void_p),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_INT = ctypes.c_int
_U32 = ctypes.c_uint32

# name -> (restype, argtypes); the list is also what the export test checks
SIGNATURES = {
    "kdn_abi_version": (_INT, []),
    "kdn_last_error": (ctypes.c_char_p, []),
    "kdn_fwht_lift": (_INT, [_P, _INT, _P, _INT, _I64, ctypes.POINTER(KdnProjection), _P]),
    "kdn_chunked_prefill_workspace_size": (ctypes.c_size_t, [_I64, _I64, _I32, _I32, ctypes.POINTER(KdnProjection), _INT]),
    "kdn_chunked_prefill": (_INT, [_P, _P, _P, _INT, _P, _P, _INT, _P, _P, _INT, _P, _I64, _I64, _I32, _I32,
                                   ctypes.POINTER(KdnProjection), _INT, _P, ctypes.c_size_t, _P]),
    "kdn_chunked_prefill_static": (_INT, [_P, _P, _P, _INT, _P, _P, _INT, _P, _P, _INT, _P, _I64, _I64, _I32, _I32,
                                          ctypes.POINTER(KdnProjection), _P]),
    "kdn_chunked_prefill_varlen": (_INT, [_P, _P, _P, _INT, _P, _P, _INT, _P, _P, _INT, _P, _P, _P, _I64, _I64, _I32,
                                          _I32, ctypes.POINTER(KdnProjection), _P]),
    "kdn_chunked_prefill_backward_workspace_size": (ctypes.c_size_t, [_I64, _I64, _I32, _I32,
                                                                       ctypes.POINTER(KdnProjection)]),
    "kdn_chunked_prefill_backward": (_INT, [_P, _P, _P, _INT, _P, _P, _INT, _P, _P, _INT, _P, _P, _P, _P, _P, _P, _P,
                                            _I64, _I64, _I32, _I32, ctypes.POINTER(KdnProjection), _P,
                                            ctypes.c_size_t, _P]),
    "kdn_set_prefill_events": (_INT, [ctypes.POINTER(ctypes.c_void_p), _INT]),
    "kdn_prefill_launch_count": (_INT, []),
    "kdn_tp_out_proj": (_INT, [_P, _P, _P, _INT, _P, _I64, _I32, _I32, _P]),
    "kdn_tp_out_proj_tiles": (_I64, [_I64, _I32]),
    "kdn_linear": (_INT, [_P, _P, _P, _INT, _I64, _I32, _I32, _I64, _P]),
    "kdn_linear_swiglu": (_INT, [_P, _P, _P, _I64, _I32, _I32, _I64, _P]),
    "kdn_anchor_qkv": (_INT, [_P, _INT, _P, _P, _P, _I64, _I64, _I32, _I32, ctypes.c_float, _P, _INT, _P, _P, _I64,
                              _I64, _P]),
    "kdn_varlen_causal_attention": (_INT, [_P, _P, _P, _INT, _P, _P, _I64, _I64, _I32, _I32, _I64, _I64, _I64, _P,
                                           _P]),
    "kdn_tp_out_proj_allreduce": (_INT, [_P, _P, _P, _P, _INT, _P, _P, _U32, _I32, _I32, _I64, _I32, _I32, _P]),
    "kdn_tp_out_proj_allreduce_peer": (_INT, [_P, _P, ctypes.POINTER(_P), _INT, ctypes.POINTER(_P), _U32, _I32, _I32,
                                              _I64, _I32, _I32, _P]),
    "kdn_ragged_transpose": (_INT, [_P, _P, _P, _INT, _I64, _I64, _I32, _I64, _INT, _P]),
    "kdn_decode_attention_workspace_size": (ctypes.c_size_t, [_I64, _I32, _I64]),
    "kdn_decode_attention": (_INT, [_P, _P, _P, _P, _P, _INT, _I64, _I32, _I64, _I32, _P, ctypes.c_size_t, _P]),
    "kdn_rmsnorm": (_INT, [_P, _INT, _P, _INT, _P, _I64, _I32, ctypes.c_float, _P]),
    "kdn_add_rmsnorm": (_INT, [_P, _P, _INT, _P, _INT, _P, _P, _I64, _I32, ctypes.c_float, _P]),
    "kdn_swiglu": (_INT, [_P, _P, _INT, _I64, _I32, _P]),
    "kdn_mixer_inputs": (_INT, [_P, _INT, _I64, _I32, _I32, _I64, _P, _INT, _P, _I64, _P, _P, _P, _P, _P, _P]),
    "kdn_copy_rows": (_INT, [_P, ctypes.c_size_t, _P, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, _P]),
    "kdn_affine_compose": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _P]),
    "kdn_affine_prefix_states": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _P]),
    "kdn_block_transition_workspace_size": (ctypes.c_size_t, [_I64, _I64, _I32, ctypes.POINTER(KdnProjection)]),
    "kdn_block_transition": (_INT, [_P, _P, _INT, _P, _P, _INT, _P, _P, _I64, _I64, _I32, _I32,
                                    ctypes.POINTER(KdnProjection), _P, ctypes.c_size_t, _P]),
    "kdn_decode_step": (_INT, [_P, _P, _P, _INT, _P, _P, _INT, _P, _INT, _I64, _P, _INT, _P, _INT, _I64, _I32, _I32,
                               ctypes.POINTER(KdnProjection), _INT, _P]),
    "kdn_fork_state": (_INT, [_P, _I64, _I64, _I64, _I64, _P]),
    "kdn_device_error": (_INT, [_P, ctypes.POINTER(_INT)]),
}

_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH):
    """Load libkdn.so once and attach signatures; raises if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"libkdn.so not found at {path}: build it with `python kernel-deltanet_b200/build.py` "
                "(kdn_b200 has no CPU fallback)")
        try:
            import torch  # noqa: F401  (load torch's CUDA libraries first)
        except ImportError:
            pass
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.kdn_abi_version() != ABI_VERSION:
            raise RuntimeError(f"libkdn ABI {lib.kdn_abi_version()} != expected {ABI_VERSION}")
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != KDN_OK:
        msg = load().kdn_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({_ERR_NAMES.get(rc, rc)}): {msg}")


def dtype_code(t) -> int:
    import torch

    if t.dtype == torch.float32:
        return KDN_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return KDN_DTYPE_BF16
    raise RuntimeError(f"unsupported dtype {t.dtype}: libkdn takes float32 or bfloat16")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream
