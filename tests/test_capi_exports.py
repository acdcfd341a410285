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


@pytest.fixture(scope="module")
def lib():
    from kdn_b200 import _lib

    return _lib.load()


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


def test_prefill_event_hook_argument_checks(lib):
    assert lib.kdn_set_prefill_events(None, 1) == 1
    assert lib.kdn_set_prefill_events(None, 0) == 0
    assert lib.kdn_prefill_launch_count() == 0
