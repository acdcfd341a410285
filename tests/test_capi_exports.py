"""CPU checks of the C ABI: the library loads, exports what include/kdn.h
declares, and rejects bad arguments with status codes (no kernel launches)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "kdn.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kdn_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("kdn_fwht_lift", "kdn_chunked_prefill", "kdn_decode_step", "kdn_fork_state", "kdn_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in _declared():
        assert hasattr(lib, name), f"libkdn.so does not export {name}"


def test_binding_covers_header():
    from kdn_b200 import _lib

    assert sorted(_lib.SIGNATURES) == _declared()


def test_abi_version(lib):
    from kdn_b200 import _lib

    assert lib.kdn_abi_version() == _lib.ABI_VERSION


def _proj(d_k=64, D=512, phase=8):
    from kdn_b200 import _lib

    p = _lib.KdnProjection()
    p.d_k, p.D, p.tau_inv, p.amp, p.phase = d_k, D, 0.35, 0.0625, phase
    return p


def test_rejects_unsupported_dk(lib):
    from kdn_b200 import _lib

    rc = lib.kdn_fwht_lift(8, 0, 8, 0, 4, _proj(d_k=128), None)
    assert rc == 2
    assert b"d_k=128" in lib.kdn_last_error()


def test_rejects_bad_D_and_null_phase(lib):
    assert lib.kdn_fwht_lift(8, 0, 8, 0, 4, _proj(D=520), None) == 2
    assert lib.kdn_fwht_lift(8, 0, 8, 0, 4, _proj(phase=0), None) == 1


def test_prefill_argument_checks(lib):
    p = _proj()
    args = lambda **kw: dict(dict(q=8, k=8, v=8, ind=0, beta=8, decay=None, gd=0, s0=None, y=8, yd=0, s=8,
                                  N=1, T=64, dv=64, C=64, mode=0, ws=256, wsb=1 << 40), **kw)

    def call(a):
        return lib.kdn_chunked_prefill(a["q"], a["k"], a["v"], a["ind"], a["beta"], a["decay"], a["gd"], a["s0"],
                                       a["y"], a["yd"], a["s"], a["N"], a["T"], a["dv"], a["C"], p, a["mode"],
                                       a["ws"], a["wsb"], None)

    assert call(args(C=48)) == 2
    assert call(args(dv=24)) == 2
    assert call(args(mode=7)) == 1
    assert call(args(N=0)) == 1
    assert call(args(s=None)) == 1
    assert call(args(wsb=16)) == 4
    assert b"workspace" in lib.kdn_last_error()


def test_workspace_size_positive(lib):
    assert lib.kdn_chunked_prefill_workspace_size(16, 65536, 64, 64, _proj(), 0) > 0
    assert lib.kdn_chunked_prefill_workspace_size(16, 65536, 64, 48, _proj(), 0) == 0


def test_decode_argument_checks(lib):
    p = _proj()
    base = [8, 8, 8, 0, 8, None, 0, 8, 0, 4, 8, 1, 8, 0, 2, 16, 64, p, 0, None]
    bad_idx = list(base); bad_idx[11] = 5
    assert lib.kdn_decode_step(*bad_idx) == 1
    bad_ro = list(base); bad_ro[18] = 3
    assert lib.kdn_decode_step(*bad_ro) == 1
    bad_dv = list(base); bad_dv[16] = 40
    assert lib.kdn_decode_step(*bad_dv) == 2
    zero_tok = list(base); zero_tok[14] = 0
    assert lib.kdn_decode_step(*zero_tok) == 0


def test_fork_argument_checks(lib):
    assert lib.kdn_fork_state(8, 4, 1024, 0, 4, None) == 1
    assert lib.kdn_fork_state(8, 4, 1024, -1, 2, None) == 1
    assert lib.kdn_fork_state(None, 4, 1024, 0, 1, None) == 1
    assert lib.kdn_fork_state(8, 4, 1024, 2, 2, None) == 0  # same slot: nothing to do


def test_no_cpu_fallback():
    import torch
    from kdn_b200 import FastWalshHadamardProjection, fused_chunked_deltanet_forward

    p = FastWalshHadamardProjection()
    with pytest.raises(RuntimeError, match="CUDA"):
        p(torch.zeros(2, 64))
    x = torch.zeros(1, 8, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_chunked_deltanet_forward(x, x, x, torch.zeros(1, 8), None, p)


def test_projection_buffers_match_golden(golden_dir):
    import numpy as np
    from kdn_b200 import FastWalshHadamardProjection

    for seed in (42, 7):
        g = np.load(os.path.join(golden_dir, f"lift_seed{seed}.npz"))
        p = FastWalshHadamardProjection(64, 512, seed)
        np.testing.assert_array_equal(p.d1.numpy(), g["d1"])
        np.testing.assert_array_equal(p.d3.numpy(), g["d3"])
        np.testing.assert_array_equal(p.b.numpy(), g["b"])
        np.testing.assert_array_equal(p.Omega.numpy(), g["omega"])
        s, _ = p.kdn_projection("cpu")
        for m in range(8):
            for st, d in enumerate((g["d1"], g["d2"], g["d3"])):
                bits = sum(1 << i for i in range(64) if d[m, i] < 0)
                assert s.sign_bits[m][st] == bits


def test_projection_from_reference_buffers(golden_dir):
    """A projection built from a reference projection's d1/d2/d3/b buffers (seed 7 here, the reference's
    own draws from the golden fixture) carries the same sign bits and phase into the kdn_projection
    struct as one drawn with that seed -- and is not the default seed's projection."""
    import types

    import numpy as np
    import torch
    from kdn_b200 import FastWalshHadamardProjection

    g = np.load(os.path.join(golden_dir, "lift_seed7.npz"))
    ref = types.SimpleNamespace(d_k=64, D=512, d1=torch.from_numpy(g["d1"]), d2=torch.from_numpy(g["d2"]),
                                d3=torch.from_numpy(g["d3"]), b=torch.from_numpy(g["b"]))
    p = FastWalshHadamardProjection.from_reference(ref)
    drawn = FastWalshHadamardProjection(64, 512, 7)
    default = FastWalshHadamardProjection(64, 512, 42)
    s, ph = p.kdn_projection("cpu")
    s7, ph7 = drawn.kdn_projection("cpu")
    s42, _ = default.kdn_projection("cpu")
    bits = lambda st: [[st.sign_bits[m][i] for i in range(3)] for m in range(8)]
    assert bits(s) == bits(s7) and bits(s) != bits(s42)
    for m in range(8):
        for st, d in enumerate((g["d1"], g["d2"], g["d3"])):
            assert s.sign_bits[m][st] == sum(1 << i for i in range(64) if d[m, i] < 0)
    assert torch.equal(ph, ph7) and torch.equal(ph, torch.from_numpy(g["b"]))
    np.testing.assert_array_equal(p.Omega.numpy(), g["omega"])
    assert (s.d_k, s.D, s.tau_inv, s.amp) == (s7.d_k, s7.D, s7.tau_inv, s7.amp)


def test_prefill_event_hook_argument_checks(lib):
    assert lib.kdn_set_prefill_events(None, 1) == 1
    assert lib.kdn_set_prefill_events(None, 0) == 0
    assert lib.kdn_prefill_launch_count() == 0


def test_affine_argument_checks(lib):
    # overlapping output / input, misalignment, unsupported sizes: rejected before any launch
    assert lib.kdn_affine_compose(4096, 8192, 16384, None, 4096, 1 << 20, 1, 64, 16, None) == 1
    assert b"overlap" in lib.kdn_last_error()
    assert lib.kdn_affine_compose(4104, 8192, 16384, None, 1 << 20, 1 << 21, 1, 64, 16, None) == 1
    assert lib.kdn_affine_compose(4096, 8192, 16384, None, 1 << 20, 1 << 21, 1, 40, 16, None) == 2
    assert lib.kdn_affine_compose(4096, 8192, 16384, None, 1 << 20, 1 << 21, 0, 64, 16, None) == 1
    assert lib.kdn_affine_compose(None, None, 16384, None, None, None, 1, 64, 16, None) == 0  # nothing asked
    assert lib.kdn_affine_compose(None, 8192, 16384, None, 1 << 20, None, 1, 64, 16, None) == 1  # A1 missing
    assert lib.kdn_affine_prefix_states(4096, 1 << 20, None, 1 << 24, None, -1, 1, 64, 16, None) == 1
    assert lib.kdn_affine_prefix_states(None, None, None, 1 << 24, None, 2, 1, 64, 16, None) == 1
    # final_state overlapping the states it is computed from
    assert lib.kdn_affine_prefix_states(1 << 30, 1 << 31, None, 1 << 24, 1 << 24, 2, 1, 64, 16, None) == 1


def test_block_transition_argument_checks(lib):
    p = _proj()
    assert lib.kdn_block_transition_workspace_size(2, 130, 64, p) > 0
    assert lib.kdn_block_transition_workspace_size(2, 130, 48, p) == 0
    call = lambda **kw: lib.kdn_block_transition(
        kw.get("k", 8), kw.get("v", 8), 0, 8, None, 0, kw.get("A", 4096), kw.get("B", 8192), 2, 130,
        kw.get("dv", 64), kw.get("C", 64), p, kw.get("ws", 256), kw.get("wsb", 16), None)
    assert call() == 4
    assert b"workspace" in lib.kdn_last_error()
    assert call(C=48) == 2
    assert call(dv=24) == 2
    assert call(v=None) == 1            # B asked without values
    assert call(A=None, B=None) == 0    # nothing asked


def test_tp_out_proj_argument_checks(lib):
    assert lib.kdn_tp_out_proj(4096, 8192, 16384, 0, None, 128, 200, 64, None) == 2   # N not a multiple of 256
    assert lib.kdn_tp_out_proj(4096, 8192, 16384, 0, None, 128, 256, 48, None) == 2   # K not a multiple of 64
    assert lib.kdn_tp_out_proj(4104, 8192, 16384, 0, None, 128, 256, 64, None) == 1   # misaligned
    assert lib.kdn_tp_out_proj(4096, 8192, None, 0, None, 128, 256, 64, None) == 1    # no output
    assert lib.kdn_tp_out_proj(4096, 8192, 16384, 7, None, 128, 256, 64, None) == 1   # bad dtype
    assert lib.kdn_tp_out_proj(4096, 8192, None, 1, 16384, 128, 256, 64, None) == 2   # multicast sum is fp32
    assert lib.kdn_tp_out_proj(4096, 8192, 16384, 0, None, 0, 256, 64, None) == 0     # nothing to do


def test_tp_out_proj_allreduce_argument_checks(lib):
    P = 4096
    assert lib.kdn_tp_out_proj_tiles(300, 512) == 3 * 2
    assert lib.kdn_tp_out_proj_tiles(300, 500) == 0
    args = lambda **kw: [kw.get(n, d) for n, d in (("y", P), ("w", P), ("out", P), ("mc", P), ("dt", 0), ("fl", P),
                                                   ("flmc", P),
                                                   ("target", 2), ("rank", 0), ("world", 2), ("M", 128), ("N", 256),
                                                   ("K", 64))] + [None]
    assert lib.kdn_tp_out_proj_allreduce(*args(rank=2)) == 1          # rank outside the world
    assert lib.kdn_tp_out_proj_allreduce(*args(world=0, rank=0)) == 1
    assert lib.kdn_tp_out_proj_allreduce(*args(N=384)) == 2           # N not a multiple of 256
    assert lib.kdn_tp_out_proj_allreduce(*args(K=96)) == 2            # K not a multiple of 64
    assert lib.kdn_tp_out_proj_allreduce(*args(fl=None)) == 1         # no counters
    assert lib.kdn_tp_out_proj_allreduce(*args(mc=P + 8)) == 1        # misaligned multicast output
    assert lib.kdn_tp_out_proj_allreduce(*args(flmc=P + 2)) == 1      # misaligned counters
    assert lib.kdn_tp_out_proj_allreduce(*args(dt=3)) == 1            # bad output dtype
    assert lib.kdn_tp_out_proj_allreduce(*args(M=0)) == 0             # nothing to do


def test_tp_out_proj_allreduce_peer_argument_checks(lib):
    import ctypes

    P = 4096
    arr = lambda *v: (ctypes.c_void_p * len(v))(*v)
    call = lambda outs, ctrs, rank=0, world=2, N=256, K=64, M=128, dt=0: lib.kdn_tp_out_proj_allreduce_peer(
        P, P, outs, dt, ctrs, 2, rank, world, M, N, K, None)
    assert call(arr(P, P), arr(P, P), world=9) == 1                # more ranks than the kernel takes
    assert call(arr(P, P), arr(P, P), rank=2) == 1
    assert call(arr(P, P), arr(P, P), N=128) == 2
    assert call(arr(P, P), arr(P, P), K=32) == 2
    assert call(arr(P, None), arr(P, P)) == 1                      # a missing copy
    assert call(arr(P, P + 4), arr(P, P)) == 1                     # a misaligned copy
    assert call(None, arr(P, P)) == 1
    assert call(arr(P, P), arr(P, P), dt=5) == 1                   # bad output dtype
    assert call(arr(P, P), arr(P, P), M=0) == 0
