"""Ragged (varlen) prefill over a slot-mapped state pool.

CPU: argument checks (raised before any device work).  GPU: every sequence of a packed
batch against the oracle run from its own pool slot, fp32 (<= 1e-4) and bf16 (outputs
<= 2e-2, states <= 1e-2) modes, with fresh sequences, a zero-length sequence and runs of
equal-length sequences on consecutive slots (merged into one call).
"""

import numpy as np
import pytest
import torch

import oracle
from conftest import fro_rel, rel_err


def _batch(seed, lens, H=2, dv=64, num_slots=8, gated=True):
    rng = np.random.default_rng(seed)
    total = sum(lens)
    q = rng.standard_normal((total, H, 64)); q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((total, H, 64)); k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((total, H, dv))
    beta = 1 / (1 + np.exp(-rng.standard_normal((total, H))))
    decay = 1 / (1 + np.exp(-(rng.standard_normal((total, H)) + 3))) if gated else None
    pool = 0.1 * rng.standard_normal((num_slots, H, dv, 512))
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    return q, k, v, beta, decay, pool, cu


def test_argument_checks_cpu():
    from kdn_b200 import ragged_prefill

    q, k, v, beta, decay, pool, cu = _batch(0, [3, 5])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).float()
    args = lambda **kw: dict(dict(query=t(q), key=t(k), value=t(v), beta=t(beta), decay=t(decay),
                                  cu_seqlens=torch.tensor(cu), recurrent_states=t(pool),
                                  slot_mapping=torch.tensor([1, 4]), output=torch.empty(8, 2, 64)), **kw)
    with pytest.raises(RuntimeError, match="cu_seqlens"):
        ragged_prefill(**args(cu_seqlens=torch.tensor([0, 5, 3])))
    with pytest.raises(RuntimeError, match="cu_seqlens"):
        ragged_prefill(**args(cu_seqlens=torch.tensor([0, 3, 9])))
    with pytest.raises(RuntimeError, match="one slot"):
        ragged_prefill(**args(slot_mapping=torch.tensor([2, 2])))
    with pytest.raises(RuntimeError, match="out of range"):
        ragged_prefill(**args(slot_mapping=torch.tensor([0, 8])))
    with pytest.raises(RuntimeError, match="output"):
        ragged_prefill(**args(output=torch.empty(8, 2, 32)))
    with pytest.raises(RuntimeError, match="CUDA"):
        ragged_prefill(**args())


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_ragged_prefill_matches_oracle_per_sequence(mode):
    import kdn_b200

    dev = "cuda:0"
    lens = [1, 63, 130, 0, 64, 64, 64, 200]
    slots = [3, 0, 5, 7, 1, 2, 4, 6]   # sequences 4, 5 share a run (equal length, consecutive slots)
    fresh = [False, True, False, False, False, False, False, False]
    q, k, v, beta, decay, pool, cu = _batch(7, lens)
    dt = torch.bfloat16 if mode == "bf16" else torch.float32
    if mode == "bf16":
        q, k, v = (torch.from_numpy(a).bfloat16().double().numpy() for a in (q, k, v))
    d = lambda a, t=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).to(dev, t)
    states = d(pool)
    out = torch.empty(sum(lens), 2, 64, device=dev, dtype=dt)
    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    kdn_b200.ragged_prefill(d(q, dt), d(k, dt), d(v, dt), d(beta), d(decay), torch.tensor(cu, device=dev), states,
                            torch.tensor(slots, device=dev), out, proj, mode=mode,
                            initial_state_mask=torch.tensor([not f for f in fresh]))
    torch.cuda.synchronize()
    consts = oracle.make_projection_constants()
    y = out.float().cpu().numpy()
    S = states.cpu().numpy()
    tol_y, tol_s = (2e-2, 1e-2) if mode == "bf16" else (1e-4, 1e-4)
    for i, (T, s, f) in enumerate(zip(lens, slots, fresh)):
        a, b = cu[i], cu[i + 1]
        S0 = np.zeros((2, 64, 512)) if f else pool[s]
        if T == 0:
            assert fro_rel(S[s], S0) < 1e-7
            continue
        tr = lambda x: np.ascontiguousarray(np.swapaxes(x[a:b], 0, 1))  # [T, H, .] -> [H, T, .]
        y_ref, S_ref = oracle.chunked_deltanet_forward(tr(q), tr(k), tr(v), tr(beta), tr(decay), consts, 64, S0)
        assert rel_err(np.swapaxes(y[a:b], 0, 1), y_ref) < tol_y, i
        assert fro_rel(S[s], S_ref) < tol_s, i


@pytest.mark.gpu
def test_varlen_batch_one_launch_matches_oracle():
    """Enough (sequence, head) scans to take the one-launch varlen path (80 sequences x 2 heads >=
    SMs): lengths 0 to 300 including 1 and chunk multiples, fresh and carried states, arbitrary slots."""
    import kdn_b200
    from kdn_b200 import _lib

    dev = "cuda:0"
    rng = np.random.default_rng(21)
    nseq = 80
    lens = [int(x) for x in rng.integers(0, 300, nseq)]
    lens[:6] = [0, 1, 64, 128, 299, 0]
    slots = [int(s) for s in rng.permutation(96)[:nseq]]
    fresh = [bool(x) for x in rng.integers(0, 2, nseq)]
    q, k, v, beta, decay, pool, cu = _batch(9, lens, num_slots=96)
    q, k, v = (torch.from_numpy(a).bfloat16().double().numpy() for a in (q, k, v))
    d = lambda a, t=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).to(dev, t)
    states = d(pool)
    out = torch.empty(sum(lens), 2, 64, device=dev, dtype=torch.bfloat16)
    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    kdn_b200.load().kdn_prefill_launch_count()
    kdn_b200.ragged_prefill(d(q, torch.bfloat16), d(k, torch.bfloat16), d(v, torch.bfloat16), d(beta), d(decay),
                            torch.tensor(cu, device=dev), states, torch.tensor(slots, device=dev), out, proj,
                            mode="bf16", initial_state_mask=torch.tensor([not f for f in fresh]))
    torch.cuda.synchronize()
    assert kdn_b200.load().kdn_prefill_launch_count() == 1  # the last prefill call was the single varlen launch
    consts = oracle.make_projection_constants()
    y = out.float().cpu().numpy()
    S = states.cpu().numpy()
    for i, (T, s, f) in enumerate(zip(lens, slots, fresh)):
        a, b = cu[i], cu[i + 1]
        S0 = np.zeros((2, 64, 512)) if f else pool[s]
        if T == 0:
            assert fro_rel(S[s], S0) < 1e-7
            continue
        tr = lambda x: np.ascontiguousarray(np.swapaxes(x[a:b], 0, 1))
        y_ref, S_ref = oracle.chunked_deltanet_forward(tr(q), tr(k), tr(v), tr(beta), tr(decay), consts, 64, S0)
        assert rel_err(np.swapaxes(y[a:b], 0, 1), y_ref) < 2e-2, i
        assert fro_rel(S[s], S_ref) < 1e-2, i
    untouched = sorted(set(range(96)) - set(slots))
    assert np.array_equal(S[untouched], pool[untouched].astype(np.float32))


@pytest.mark.gpu
def test_varlen_rejects_rows_outside_the_batch():
    """A scan whose rows fall outside the tensors is not run: its state passes through and the
    device error word reports it (bounds checked in the kernel; nothing is read out of range)."""
    import kdn_b200
    from kdn_b200 import _lib

    dev = torch.device("cuda", 0)
    lib = kdn_b200.load()
    proj = kdn_b200.FastWalshHadamardProjection().to(dev)
    p, _ = proj.kdn_projection(dev)
    rows = 256
    q = torch.nn.functional.normalize(torch.randn(rows, 64, device=dev), dim=-1).bfloat16()
    v = torch.randn(rows, 64, device=dev).bfloat16()
    beta = torch.full((rows,), 0.5, device=dev)
    y = torch.zeros(rows, 64, device=dev, dtype=torch.bfloat16)
    S0 = torch.randn(2, 64, 512, device=dev)
    S = torch.empty_like(S0)
    offs = torch.tensor([0, 200], device=dev)
    lens = torch.tensor([128, 100], device=dev)  # scan 1 would read rows 200..299 of 256
    rc = lib.kdn_chunked_prefill_varlen(q.data_ptr(), q.data_ptr(), v.data_ptr(), _lib.KDN_DTYPE_BF16,
                                        beta.data_ptr(), None, _lib.KDN_DTYPE_F32, S0.data_ptr(), y.data_ptr(),
                                        _lib.KDN_DTYPE_BF16, S.data_ptr(), offs.data_ptr(), lens.data_ptr(), 2, rows,
                                        64, 64, p, _lib.stream_handle(dev))
    torch.cuda.synchronize()
    assert rc == 0
    assert torch.equal(S[1], S0[1])
    assert float(y[200:].float().abs().max()) == 0.0
    assert kdn_b200.serving.vllm_kernel_deltanet_op.device_error(dev) != 0


@pytest.mark.gpu
@pytest.mark.parametrize("cu_list", [[-1000, 10], [0, 4, -2, 10], [0, 6, 20]])
def test_ragged_transpose_leaves_malformed_rows_untouched(cu_list):
    """kdn_ragged_transpose skips every row of a sequence whose offsets are negative, decreasing or
    past the end (the C entry point does not validate cu_seqlens; the kernel guards each row):
    those rows of dst keep their contents and nothing outside the tensors is touched."""
    import kdn_b200
    from kdn_b200 import _lib

    dev = torch.device("cuda", 0)
    lib = kdn_b200.load()
    total, H, w = 10, 2, 64
    src = torch.randn(total, H, w, device=dev)
    guard = 64
    buf = torch.full((guard + total + guard, H, w), 5.0, device=dev)  # guard rows on both sides
    dst = buf[guard:guard + total]
    cu = torch.tensor(cu_list, device=dev, dtype=torch.int64)
    rc = lib.kdn_ragged_transpose(src.data_ptr(), dst.data_ptr(), cu.data_ptr(), _lib.KDN_INDEX_I64,
                                  len(cu_list) - 1, total, H, w * 4, 1, _lib.stream_handle(dev))
    torch.cuda.synchronize()
    assert rc == 0
    assert bool((buf[:guard] == 5.0).all()) and bool((buf[guard + total:] == 5.0).all())
    good = [i for i in range(len(cu_list) - 1) if 0 <= cu_list[i] <= cu_list[i + 1] <= total]
    rows = dst.reshape(-1, w)
    for i in good:  # well-formed sequences: their head-major block
        c0, c1 = cu_list[i], cu_list[i + 1]
        assert torch.equal(rows[c0 * H:c1 * H], src[c0:c1].transpose(0, 1).reshape(-1, w))
    n_written = sum((cu_list[i + 1] - cu_list[i]) * H for i in good)
    assert int((rows == 5.0).all(-1).sum()) == total * H - n_written
