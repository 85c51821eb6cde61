"""Column-parallel W4A16 linear: a decoder linear's output features split over the GPUs of one node.

The reference runs every linear on one GPU (`src/fastserve/engine/model.py:43-46,91-96`: nn.Linear, or vLLM's
Marlin kernel in production). Here the packed INT4 weight [N, K/8] (with its scales and zero points) is cut along
N into one contiguous block of N/G rows per rank: each rank reads only its N·K/G codes from HBM, runs the W4A16
kernel on them, and an all-gather over the process group (NCCL over NVLink on a B200 node) assembles y [M, N] on
every rank. Groups run along K, so cutting along N never splits a quantization group: each shard is an ordinary
W4A16 weight and the kernels take it unchanged.

For the fused gate_up + SwiGLU weight (rows alternate gate and up) the cut keeps (gate, up) pairs together, so
each rank produces silu(g) * u for its N/(2G) intermediate features and the gather assembles [M, N/2].

At decode sizes (M = 1, y a few KB) the collective is latency-bound: the gather costs more than the weight bytes
saved per rank. The layer exists for the cases that are bandwidth-bound per GPU (large N, several tokens) and to
keep a model's weights resident across GPUs; `bench.py` reports its per-call time as measured.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist
from torch import nn

LocalLinear = Callable[..., torch.Tensor]  # (x, qweight, scales, qzeros, group=...) -> y [.., N_local]


def shard_rows(n: int, world: int, rank: int, multiple: int = 16) -> tuple[int, int]:
    """Rows [start, stop) of rank `rank` when n output rows are cut into `world` equal contiguous blocks.

    Each block must be a whole number of `multiple` rows (16: the row tile of the streaming GEMV, so a shard takes the
    same kernel as the full weight; 2 for gate/up pairs at least)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if n % (world * multiple):
        raise ValueError(f"{n} rows do not split into {world} blocks of a multiple of {multiple} rows")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_w4a16(qweight: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor | None, world: int, rank: int,
                multiple: int = 16):
    """This rank's rows of a packed W4A16 weight: (qweight, scales, qzeros) views of rows [start, stop), made
    contiguous. Every per-row tensor is cut the same way (codes, fp16 scales, packed zero points)."""
    start, stop = shard_rows(qweight.shape[0], world, rank, multiple)
    pick = lambda t: None if t is None else t[start:stop].contiguous()  # noqa: E731
    return pick(qweight), pick(scales), pick(qzeros)


class ColumnParallelW4A16Linear(nn.Module):
    """y = x . W^T with W's output rows split over `process_group`; every rank returns the full y [..., N].

    `local_linear` computes this rank's [M, N_local] block (default: `w4a16_linear`, or `w4a16_gate_up_silu` with
    `gate_up=True`); the gather is one `all_gather_into_tensor` of [M, N_local] blocks."""

    def __init__(self, qweight, scales, qzeros, group: int = 128, *, process_group=None, gate_up: bool = False,
                 local_linear: LocalLinear | None = None, full: bool = True):
        super().__init__()
        self.pg = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        if full:  # given the whole weight: keep this rank's rows
            qweight, scales, qzeros = shard_w4a16(qweight, scales, qzeros, self.world, self.rank,
                                                  32 if gate_up else 16)
        self.register_buffer("qweight", qweight)
        self.register_buffer("scales", scales)
        self.register_buffer("qzeros", qzeros)
        self.group, self.gate_up = group, gate_up
        self.in_features = qweight.shape[1] * 8
        self.local_out = qweight.shape[0] // 2 if gate_up else qweight.shape[0]
        self.out_features = self.local_out * self.world
        if local_linear is None:
            from bpt_b200.kernels.w4a16 import w4a16_gate_up_silu, w4a16_linear

            local_linear = w4a16_gate_up_silu if gate_up else w4a16_linear
        self.local_linear = local_linear

    def forward(self, x: torch.Tensor, *, out: torch.Tensor | None = None,
                local_out: torch.Tensor | None = None) -> torch.Tensor:
        """x [..., K] -> y [..., N]. `out` ([..., N], contiguous) and `local_out` ([M, N_local]) are optional
        preallocated buffers (for graph capture)."""
        lead = x.shape[:-1]
        rows = x.reshape(-1, x.shape[-1])
        m = rows.shape[0]
        if local_out is None:
            local_out = torch.empty((m, self.local_out), dtype=x.dtype, device=x.device)
        part = self.local_linear(rows, self.qweight, self.scales, self.qzeros, group=self.group, out=local_out)
        if self.world == 1:
            y = part if out is None else out.reshape(m, self.out_features).copy_(part)
            return y.reshape(*lead, self.out_features)
        blocks = torch.empty((self.world * m, self.local_out), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(blocks, part.contiguous(), group=self.pg)
        # blocks[r * m + i] = rank r's columns of token i -> y[i, r * N_local : (r + 1) * N_local]
        y = blocks.view(self.world, m, self.local_out).transpose(0, 1).reshape(m, self.out_features)
        if out is not None:
            out.reshape(m, self.out_features).copy_(y)
            y = out
        return y.reshape(*lead, self.out_features)
