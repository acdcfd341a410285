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
