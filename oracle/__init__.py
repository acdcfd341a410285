"""CPU oracle for the Kernel-DeltaNet hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithm of the path

    FWHT feature lift (kernels/fwht.py)
      -> exact gated delta-rule chunked prefill (kernels/fused_kernel_deltanet.py)
      -> single-token decode recurrence (kernels/kernel_deltanet_fused.py:288-300,
         tests/test_fused_kernel.py:33-67)

of jatin-yadav-acad/kernel-deltanet.  Every function cites the reference
file:line it follows.  It is pinned against golden vectors produced by running
the reference itself (tests/golden/make_golden.py; fixtures under
tests/golden/) -- see tests/test_oracle_golden.py.

Only tests/, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of bench.py may import this package, and only as
the checker or as the timed CPU baseline.  The product path
(``kdn_b200`` + ``libkdn.so``) never imports it.
"""

from .projection import ProjectionConstants, make_projection_constants, build_omega, lift
from .chunked import chunked_deltanet_forward
from .recurrence import token_recurrence, decode_step, decode_step_post
from .affine import compose, chunk_block_transition, apply_transition
from . import hybrid_lm

__all__ = [
    "ProjectionConstants",
    "make_projection_constants",
    "build_omega",
    "lift",
    "chunked_deltanet_forward",
    "token_recurrence",
    "decode_step",
    "decode_step_post",
    "compose",
    "chunk_block_transition",
    "apply_transition",
]
