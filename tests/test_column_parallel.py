"""The column-parallel W4A16 linear's host logic on CPU: two gloo ranks each hold half of a packed INT4 weight's
output rows, compute their block and all-gather it; every rank must end with the full y of the unsharded weight.

The per-rank block is computed by the oracle (injected as `local_linear`: no GPU here); on a B200 node the same
module runs the W4A16 kernels and NCCL (tests/test_gpu_column_parallel.py)."""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_local(gate_up: bool):
    from oracle import w4a16 as ow4

    def run(x, qweight, scales, qzeros, group=128, out=None):
        fn = ow4.w4a16_gate_up_silu if gate_up else ow4.w4a16_linear
        y = fn(x, qweight, scales, qzeros, group)
        return y if out is None else out.copy_(y)

    return run


def _weights(n, k, seed):
    from oracle import w4a16 as ow4

    w = torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.02
    return ow4.pack_w4a16(*ow4.quantize_w4a16(w, 128))


def _rank_main(rank: int, world: int, port: int, results):
    for p in (ROOT, ROOT / "bytes-per-token_b200"):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bpt_b200.column_parallel import ColumnParallelW4A16Linear
        from oracle import w4a16 as ow4

        out = {}
        for gate_up in (False, True):
            n, k = 256, 512
            qweight, scales, qzeros = _weights(n, k, seed=5)
            layer = ColumnParallelW4A16Linear(qweight, scales, qzeros, 128, gate_up=gate_up,
                                              local_linear=_oracle_local(gate_up))
            assert layer.qweight.shape[0] == n // world  # this rank reads only its rows
            for m in (1, 3):
                x = torch.randn(2, m, k, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16)
                got = layer(x)
                fn = ow4.w4a16_gate_up_silu if gate_up else ow4.w4a16_linear
                want = fn(x.reshape(-1, k), qweight, scales, qzeros, 128).reshape(2, m, -1)
                out[(gate_up, m)] = bool(torch.equal(got, want))
        results[rank] = out
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_the_full_output():
    world = 2
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.spawn(_rank_main, args=(world, _free_port(), results), nprocs=world, join=True)
    for rank in range(world):
        assert results[rank] and all(results[rank].values()), results[rank]


def test_one_process_is_the_plain_linear():
    for p in (ROOT, ROOT / "bytes-per-token_b200"):
        sys.path.insert(0, str(p))
    from bpt_b200.column_parallel import ColumnParallelW4A16Linear
    from oracle import w4a16 as ow4

    qweight, scales, qzeros = _weights(64, 256, seed=1)
    layer = ColumnParallelW4A16Linear(qweight, scales, qzeros, 128, local_linear=_oracle_local(False))
    x = torch.randn(4, 256).to(torch.bfloat16)
    assert torch.equal(layer(x), ow4.w4a16_linear(x, qweight, scales, qzeros, 128))


def test_shards_are_whole_row_tiles():
    sys.path.insert(0, str(ROOT / "bytes-per-token_b200"))
    from bpt_b200.column_parallel import shard_rows, shard_w4a16

    assert shard_rows(6144, 8, 3) == (2304, 3072)
    with pytest.raises(ValueError):
        shard_rows(6144 + 16, 8, 0)  # 6160 / 8 = 770 rows: not a multiple of the 16-row tile
    q = torch.arange(64 * 4, dtype=torch.int32).view(64, 4)
    s = torch.arange(64 * 2, dtype=torch.float16).view(64, 2)
    qw, sc, qz = shard_w4a16(q, s, None, 2, 1)
    assert torch.equal(qw, q[32:]) and torch.equal(sc, s[32:]) and qz is None
