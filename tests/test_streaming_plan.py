"""Segment plan of the streamed host prefill (`fused_chunked_deltanet_forward` with host tensors): the
sequence is covered once, in order, by segments of whole chunks (only the last may end on a partial
chunk), with short ramps at both ends and `seg`-token segments between.  Host logic only (no device)."""

import pytest

from kdn_b200.kernels.fused_kernel_deltanet import _segment_plan


@pytest.mark.parametrize("T,seg,chunk", [(65536, 8192, 64), (65536, 16384, 64), (1000, 256, 64), (1000, 192, 64),
                                         (1000, 512, 64), (517, 64, 64), (100, 64, 64), (64, 64, 64), (1, 64, 64),
                                         (4096, 1024, 32), (65536 + 37, 8192, 64)])
def test_plan_covers_the_sequence_in_whole_chunks(T, seg, chunk):
    plan = _segment_plan(T, seg, chunk)
    assert plan[0][0] == 0 and plan[-1][1] == T
    for (a0, a1), (b0, b1) in zip(plan, plan[1:]):
        assert a1 == b0  # contiguous, in order
    for t0, t1 in plan:
        assert t0 % chunk == 0 and t1 > t0
        assert t1 - t0 <= max(seg, chunk)
    for t0, t1 in plan[:-1]:  # only the last segment may end inside a chunk
        assert (t1 - t0) % chunk == 0


def test_plan_ramps_at_both_ends():
    sizes = [t1 - t0 for t0, t1 in _segment_plan(65536, 8192, 64)]
    assert sizes[:4] == [1024, 2048, 4096, 8192]
    assert sizes[-3:] == [4096, 2048, 1024]
    assert max(sizes) == 8192 and sum(sizes) == 65536


def test_plan_short_sequences_and_empty():
    assert _segment_plan(0, 8192, 64) == []
    assert _segment_plan(300, 8192, 64) == [(0, 300)]  # one (ragged) segment
    assert [t1 - t0 for t0, t1 in _segment_plan(8192 * 2, 8192, 64)] == [8192] * 2  # too short for ramps
