"""Multi-rank host logic of kdn_b200.distributed.

CPU: world_size-2 and -3 gloo process groups (spawned ranks) run the
sequence-parallel orchestration with host-side block maps and check every rank's
block against the oracle's single pass; shard_range is checked directly.
GPU (2 devices): the same orchestration through libkdn over NCCL.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import _dist_workers as W


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world, tmp_path, *extra):
    path = str(tmp_path / "result")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, path) + extra) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    results = []
    for r in range(world):
        f = f"{path}.{r}"
        results.append(open(f).read() if os.path.exists(f) else "missing")
    return results


def test_shard_range_partitions():
    from kdn_b200.distributed import shard_range

    for n in (0, 1, 7, 16, 512, 1001):
        for world in (1, 2, 3, 8):
            parts = [shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_single_process_passthrough():
    from kdn_b200 import distributed as kd

    S0 = torch.ones(1, 16, 16)
    assert kd.entering_state(torch.eye(16)[None], torch.zeros(1, 16, 16), S0) is S0
    assert kd.max_over_ranks(3.25) == 3.25


@pytest.mark.parametrize("world", [2, 3])
def test_sequence_parallel_orchestration_gloo(tmp_path, world):
    assert _run(W.gloo_sequence_parallel, world, tmp_path) == ["ok"] * world


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_sequence_parallel_prefill_nccl(tmp_path, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    assert _run(W.nccl_sequence_parallel, 2, tmp_path, mode) == ["ok", "ok"]
