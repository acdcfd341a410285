"""Generate golden vectors by running the REFERENCE implementation on CPU.

Run once in a container where the reference checkout is available:

    python tests/golden/make_golden.py /path/to/kernel-deltanet [--only-backward]

It imports the reference's own modules

    kernels/fwht.py                     FastWalshHadamardProjection
    kernels/fused_kernel_deltanet.py    fused_chunked_deltanet_forward, FusedKernelDeltaNetFunction
    kernels/blelloch_scan.py            compose_transitions
    tests/test_fused_kernel.py          sequential_deltanet_reference
    benchmarks/run_full_batch_decoding.py  step_recurrent_state

and writes the inputs and outputs of small seeded cases to ``*.npz`` files
beside this script.  The fixtures travel with the repository; nothing at test
time reads the reference.  Inputs are drawn with numpy's PCG64 generator so the
cases are reproducible; outputs are the reference's fp32 results.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _inputs(seed, N, T, d_k, dv, gated, init_state, D=512):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((N, T, d_k)).astype(np.float32)
    k = rng.standard_normal((N, T, d_k)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((N, T, dv)).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((N, T))))).astype(np.float32)
    if gated:
        decay = (1.0 / (1.0 + np.exp(-(rng.standard_normal((N, T)) + 3.0)))).astype(np.float32)
    else:
        decay = np.ones((N, T), np.float32)
    S0 = (0.1 * rng.standard_normal((N, dv, D))).astype(np.float32) if init_state else None
    return q, k, v, beta, decay, S0


PREFILL_CASES = {
    # name: (seed, N, T, d_k, dv, C, gated, init_state)
    "prefill_t130_gated_s0": (1, 1, 130, 64, 64, 64, True, True),
    "prefill_t63": (2, 1, 63, 64, 64, 64, False, False),
    "prefill_t64": (3, 1, 64, 64, 64, 64, False, False),
    "prefill_t1": (4, 1, 1, 64, 64, 64, True, True),
    "prefill_c32_dv128_gated": (5, 1, 96, 64, 128, 32, True, False),
    "prefill_t256_c64": (6, 1, 256, 64, 64, 64, False, False),
}


BACKWARD_CASES = {
    # name: (seed, N, T, d_k, dv, C, gated)
    "backward_t130_gated": (21, 1, 130, 64, 64, 64, True),
    "backward_t63_n2": (22, 2, 63, 64, 64, 64, False),
    "backward_c32_dv128_gated": (23, 1, 96, 64, 128, 32, True),
}


def backward_fixtures(ref_root: str) -> None:
    """Gradients from the reference's autograd Function (kernels/fused_kernel_deltanet.py:158-179):
    recompute the forward under autograd, then d(Y . dY)/d(q, k, v, beta, decay), fp32 on CPU."""
    sys.path.insert(0, ref_root)
    import torch

    torch.set_num_threads(1)
    from kernels.fwht import FastWalshHadamardProjection
    from kernels.fused_kernel_deltanet import FusedKernelDeltaNetFunction

    p = FastWalshHadamardProjection(64, 512, seed=42)
    for name, (seed, N, T, d_k, dv, C, gated) in BACKWARD_CASES.items():
        q, k, v, beta, decay, _ = _inputs(seed, N, T, d_k, dv, gated, False)
        dY = np.random.default_rng(seed + 1000).standard_normal((N, T, dv)).astype(np.float32)
        ins = [torch.from_numpy(a).requires_grad_(True) for a in (q, k, v, beta, decay)]
        Y = FusedKernelDeltaNetFunction.apply(*ins, p, C)
        Y.backward(torch.from_numpy(dY))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), q=q, k=k, v=v, beta=beta, decay=decay, dY=dY,
                            Y=Y.detach().numpy(), dq=ins[0].grad.numpy(), dk=ins[1].grad.numpy(),
                            dv=ins[2].grad.numpy(), dbeta=ins[3].grad.numpy(), ddecay=ins[4].grad.numpy(),
                            meta=np.array([seed, N, T, d_k, dv, C, int(gated)]))


def main(ref_root: str) -> None:
    backward_fixtures(ref_root)
    sys.path.insert(0, ref_root)
    import torch

    torch.set_num_threads(1)
    from kernels.fwht import FastWalshHadamardProjection
    from kernels.fused_kernel_deltanet import fused_chunked_deltanet_forward
    from kernels.blelloch_scan import compose_transitions

    # 1. projection constants and lift outputs (kernels/fwht.py)
    for seed in (42, 7):
        p = FastWalshHadamardProjection(64, 512, seed=seed)
        rng = np.random.default_rng(100 + seed)
        x = rng.standard_normal((16, 64)).astype(np.float32)
        x /= np.linalg.norm(x, axis=-1, keepdims=True)
        with torch.no_grad():
            phi = p(torch.from_numpy(x)).numpy()
        np.savez_compressed(
            os.path.join(HERE, f"lift_seed{seed}.npz"),
            d1=p.d1.numpy().astype(np.int8), d2=p.d2.numpy().astype(np.int8), d3=p.d3.numpy().astype(np.int8),
            b=p.b.numpy(), omega=p.Omega.numpy(), x=x, phi=phi,
        )

    # 2. chunked prefill (kernels/fused_kernel_deltanet.py:31-155), fp32
    p = FastWalshHadamardProjection(64, 512, seed=42)
    for name, (seed, N, T, d_k, dv, C, gated, init) in PREFILL_CASES.items():
        q, k, v, beta, decay, S0 = _inputs(seed, N, T, d_k, dv, gated, init)
        with torch.no_grad():
            Y, S = fused_chunked_deltanet_forward(
                torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
                torch.from_numpy(beta), torch.from_numpy(decay), p, chunk_size=C,
                initial_state=None if S0 is None else torch.from_numpy(S0),
            )
        arrays = dict(q=q, k=k, v=v, beta=beta, decay=decay, Y=Y.numpy(), S=S.numpy(),
                      meta=np.array([seed, N, T, d_k, dv, C, int(gated), int(init)]))
        if S0 is not None:
            arrays["S0"] = S0
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)

    # 3. float64 token recurrence (tests/test_fused_kernel.py:33-67)
    sys.path.insert(0, os.path.join(ref_root, "tests"))
    import test_fused_kernel as tfk

    tfk.DEVICE = torch.device("cpu")
    q, k, v, beta, decay, _ = _inputs(11, 2, 40, 64, 64, True, False)
    with torch.no_grad():
        Yr, Sr = tfk.sequential_deltanet_reference(
            torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
            torch.from_numpy(beta), torch.from_numpy(decay), p)
    np.savez_compressed(os.path.join(HERE, "recurrence_t40.npz"), q=q, k=k, v=v, beta=beta,
                        decay=decay, Y=Yr.numpy(), S=Sr.numpy())

    # 4. post-update decode step (benchmarks/run_full_batch_decoding.py:27-55)
    sys.path.insert(0, os.path.join(ref_root, "benchmarks"))
    import run_full_batch_decoding as rfbd

    rng = np.random.default_rng(12)
    B, H = 1, 2
    S_prev = (0.02 * rng.standard_normal((B, H, 64, 512))).astype(np.float32)
    qd = rng.standard_normal((B, H, 64)).astype(np.float32)
    kd = rng.standard_normal((B, H, 64)).astype(np.float32)
    qd /= np.linalg.norm(qd, axis=-1, keepdims=True)
    kd /= np.linalg.norm(kd, axis=-1, keepdims=True)
    vd = rng.standard_normal((B, H, 64)).astype(np.float32)
    bd = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, H))))).astype(np.float32)
    dd = (1.0 / (1.0 + np.exp(-(rng.standard_normal((B, H)) + 3.0)))).astype(np.float32)
    with torch.no_grad():
        yd, Sd = rfbd.step_recurrent_state(
            torch.from_numpy(qd), torch.from_numpy(kd), torch.from_numpy(vd),
            torch.from_numpy(bd), torch.from_numpy(dd), torch.from_numpy(S_prev), p)
    np.savez_compressed(os.path.join(HERE, "decode_post_step.npz"), S_prev=S_prev, q=qd, k=kd, v=vd,
                        beta=bd, decay=dd, y=yd.numpy(), S=Sd.numpy())

    # 5. affine composition (kernels/blelloch_scan.py:42-56)
    rng = np.random.default_rng(13)
    A1 = rng.standard_normal((2, 8, 8)); B1 = rng.standard_normal((2, 4, 8))
    A2 = rng.standard_normal((2, 8, 8)); B2 = rng.standard_normal((2, 4, 8))
    An, Bn = compose_transitions((torch.from_numpy(A1), torch.from_numpy(B1)),
                                 (torch.from_numpy(A2), torch.from_numpy(B2)))
    np.savez_compressed(os.path.join(HERE, "compose.npz"), A1=A1, B1=B1, A2=A2, B2=B2,
                        A=An.numpy(), B=Bn.numpy())
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    root = args[0] if args else os.environ.get("KDN_REFERENCE_ROOT", "")
    if "--only-backward" in sys.argv:
        backward_fixtures(root)
    else:
        main(root)
