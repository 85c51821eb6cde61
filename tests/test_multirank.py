"""bench.py's multi-rank host logic on CPU: two gloo ranks, each with its own measurements, must agree on the
whole-job figures (slowest rank's device time, every rank's bytes and decode tokens) exactly as the NCCL run on
the GPU box combines them. No GPU and no collective on a data path: gather_ranks only moves the small dicts."""

import os
import socket
import sys
from pathlib import Path

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, results):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        local = {
            "total_ms": 10.0 + rank,  # rank 1 is the slow one
            "e2e_ms": 20.0 - rank,
            "bytes": 1000 * (rank + 1),
            "decode_ms": 5.0 * (rank + 1),
            "decode_tokens": 64 * 20,
            "decode_bytes": 7 * (rank + 1),
        }
        gathered = bench.gather_ranks(local, dist)
        results[rank] = (gathered, bench.combine_ranks(gathered))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_combine_like_the_gpu_run():
    world = 2
    manager = mp.get_context("spawn").Manager()  # no fork of a process that already runs torch threads
    results = manager.dict()
    mp.spawn(_rank_main, args=(world, _free_port(), results), nprocs=world, join=True)
    for rank in range(world):
        gathered, whole = results[rank]
        assert [g["bytes"] for g in gathered] == [1000, 2000]  # rank order on every rank
        assert whole["total_ms"] == 11.0  # the slowest rank's device time
        assert whole["e2e_ms"] == 20.0
        assert whole["bytes"] == 3000  # every rank's work
        assert whole["decode_ms"] == 10.0
        assert whole["decode_tokens"] == 2 * 64 * 20
        assert whole["decode_bytes"] == 21


def test_one_process_needs_no_group():
    sys.path.insert(0, str(ROOT))
    import bench

    local = {"total_ms": 3.0, "e2e_ms": 4.0, "bytes": 5}
    gathered = bench.gather_ranks(local, None)
    assert gathered == [local]
    assert bench.combine_ranks(gathered) == {"total_ms": 3.0, "e2e_ms": 4.0, "bytes": 5}
