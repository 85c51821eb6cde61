"""The column-parallel W4A16 linear on two GPUs (NCCL): each rank runs the W4A16 kernel on its half of the output
rows and the all-gather assembles y. At M <= 8 (the streaming GEMV: each output row's sum is computed the same way
whatever N is) the gathered y equals the one-GPU kernel's output on the whole weight bit for bit; at M = 64 (the
tcgen05 GEMM, whose K split depends on N) it is compared with the oracle at atol / rtol 1e-2.

Needs two GPUs; skipped otherwise. The ranks are child processes with a short process-group timeout."""

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, results):
    for p in (ROOT, ROOT / "bytes-per-token_b200"):
        sys.path.insert(0, str(p))
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from bpt_b200.column_parallel import ColumnParallelW4A16Linear
        from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_gate_up_silu, w4a16_linear
        from oracle import w4a16 as ow4

        out = {}
        w = (torch.randn(6144, 2048, generator=torch.Generator().manual_seed(0)) * 0.02).to(dev)
        full = quantize_w4a16(w, 128)
        for gate_up in (False, True):
            layer = ColumnParallelW4A16Linear(*full, 128, gate_up=gate_up)
            one_gpu = w4a16_gate_up_silu if gate_up else w4a16_linear
            for m in (1, 4, 64):
                x = torch.randn(m, 2048, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16).to(dev)
                got = layer(x)
                if m <= 8:
                    out[(gate_up, m)] = bool(torch.equal(got, one_gpu(x, *full)))
                else:
                    fn = ow4.w4a16_gate_up_silu if gate_up else ow4.w4a16_linear
                    want = fn(x.cpu(), *[t.cpu() for t in full], 128, dense_bf16=True)
                    out[(gate_up, m)] = bool(torch.allclose(got.cpu().float(), want.float(), atol=1e-2, rtol=1e-2))
        torch.cuda.synchronize()
        results[rank] = out
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_column_parallel_on_two_gpus_gathers_the_one_gpu_result():
    import torch.multiprocessing as mp

    world = 2
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_rank_main, args=(world, _free_port(), results), nprocs=world, join=True)
    for rank in range(world):
        assert results[rank] and all(results[rank].values()), results[rank]
