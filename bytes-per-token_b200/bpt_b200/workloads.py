"""Seeded synthetic inputs for the benchmark configurations, and their algorithmic byte counts.

No dataset is involved anywhere on this path: every input is drawn from seeded generators with the shapes and
distributions of the configurations (the reference seeds with torch.Generator().manual_seed, seed 0 unless
swept: tests/kernels/test_kernels_gpu.py:20-22, experiments/m7.py:64-66).

    1  W4A16 GEMV, Qwen3-1.7B up_proj: x ~ N(0,1) bf16 [1, 2048], W ~ N(0, 0.02) [6144, 2048], asym INT4 g128
    2  paged FP8 decode attention: B 32, 16 Q / 8 KV heads, D 128, lengths ~ U[512, 4096], page 16,
       block table a random permutation of a 16,384-page pool; K, V ~ N(0,1), E4M3 with a per-tensor scale
    3  long-context INT8 decode attention: B 8, length 32,768 each, symmetric INT8 with an fp16 scale per
       (token, KV head), page 16, random block table
    4  W4A16 sweep over the Qwen3-1.7B decoder linears at M in {1, 4, 16, 64, 256}

Byte counts follow the roofline convention: every input once, every output once, INT4 zero-points at 4 bits
(IntSpec.bits_per_weight, quant/rtn.py:53-56).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from bpt_b200.kernels.kv_attention import PagedQuantKV
from bpt_b200.kernels.kv_write import quantize_kv_paged
from bpt_b200.kernels.w4a16 import quantize_w4a16

FP8_SCALE = 1.0 / 64.0  # per-tensor E4M3 scale for N(0,1) data: 448 * s = 7 standard deviations

QWEN3_1_7B = {
    "hidden": 2048,
    "intermediate": 6144,
    "layers": 28,
    "q_heads": 16,
    "kv_heads": 8,
    "head_dim": 128,
    "vocab": 151936,
    "rope_theta": 1e6,
    "eps": 1e-6,
}

# Config 4: every decoder linear of Qwen3-1.7B as (name, N, K); gate_up is the fused pair.
SWEEP_LINEARS = [
    ("q_proj", 2048, 2048),
    ("k_proj", 1024, 2048),
    ("v_proj", 1024, 2048),
    ("o_proj", 2048, 2048),
    ("gate_up", 12288, 2048),
    ("down_proj", 2048, 6144),
]
SWEEP_M = (1, 4, 16, 64, 256)


def w4a16_bytes(m: int, n: int, k: int, group: int = 128) -> int:
    """Codes + fp16 scales + 4-bit zero-points + bf16 x + bf16 y."""
    g = k // group
    return n * k // 2 + n * g * 2 + n * g // 2 + 2 * m * k + 2 * m * n


def paged_bytes(lengths: torch.Tensor, q_heads: int, kv_heads: int, head_dim: int, kind: str, block_size: int = 16,
                out_bytes: int = 2) -> int:
    """KV bytes of every visible token (K and V, scales for INT8) + block-table entries + q (bf16) + out."""
    total = int(lengths.to(torch.int64).sum())
    pages = int(((lengths.to(torch.int64) + block_size - 1) // block_size).sum())
    per_token = 2 * kv_heads * head_dim + (2 * kv_heads * 2 if kind == "int8" else 0)
    b = lengths.numel()
    return total * per_token + 4 * pages + b * q_heads * head_dim * 2 + b * q_heads * head_dim * out_bytes


@dataclass
class W4A16Case:
    x: torch.Tensor  # bf16 [M, K]
    qweight: torch.Tensor
    scales: torch.Tensor
    qzeros: torch.Tensor
    group: int
    w: torch.Tensor | None = None  # the dense fp32 weight on the CPU, when kept

    @property
    def bytes(self) -> int:
        return w4a16_bytes(self.x.shape[0], self.qweight.shape[0], self.x.shape[1], self.group)


def w4a16_case(m: int, n: int, k: int, group: int = 128, seed: int = 0, device="cuda", keep_dense: bool = False):
    """x ~ N(0,1) bf16 [m, k]; W ~ N(0, 0.02) [n, k] quantized on the GPU to asymmetric INT4."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    qweight, scales, qzeros = quantize_w4a16(w.to(device), group)
    return W4A16Case(x.to(device), qweight, scales, qzeros, group, w if keep_dense else None)


@dataclass
class PagedCase:
    q: torch.Tensor  # bf16 [B, Hq, D]
    kv: PagedQuantKV
    lengths: torch.Tensor  # int32 [B]
    q_heads: int

    @property
    def bytes(self) -> int:
        return paged_bytes(self.lengths.cpu(), self.q_heads, self.kv.kv_heads, self.kv.head_dim, self.kv.kind,
                           self.kv.block_size)

    @property
    def max_length(self) -> int:
        return int(self.lengths.max())


def block_table_for(lengths: torch.Tensor, block_size: int, num_blocks: int, generator: torch.Generator,
                    width: int | None = None) -> torch.Tensor:
    """Each sequence's pages drawn, without replacement, from a random permutation of the pool."""
    need = ((lengths.to(torch.int64) + block_size - 1) // block_size).tolist()
    width = width or max(max(need), 1)
    if sum(need) > num_blocks:
        raise ValueError(f"{sum(need)} pages needed, the pool has {num_blocks}")
    perm = torch.randperm(num_blocks, generator=generator)
    table = torch.empty(len(need), width, dtype=torch.int32)
    pos = 0
    spare = perm[sum(need):] if sum(need) < num_blocks else perm
    for i, n in enumerate(need):
        table[i, :n] = perm[pos : pos + n].to(torch.int32)
        pos += n
        if width > n:  # entries past the sequence's end: valid pages, never read
            table[i, n:] = spare[torch.arange(width - n) % spare.numel()].to(torch.int32)
    return table


def fill_pool(kv: PagedQuantKV, seed: int, chunk_blocks: int = 2048) -> None:
    """Draw K, V ~ N(0,1) for every slot of the pool and store them through the write kernel."""
    nb, bs, hkv, d = kv.k_pool.shape
    device = kv.k_pool.device
    g = torch.Generator(device=device).manual_seed(seed)
    offsets = torch.arange(bs, dtype=torch.int32, device=device)
    for start in range(0, nb, chunk_blocks):
        n = min(chunk_blocks, nb - start)
        k = torch.randn(n, hkv, bs, d, generator=g, device=device).to(torch.bfloat16)
        v = torch.randn(n, hkv, bs, d, generator=g, device=device).to(torch.bfloat16)
        blocks = torch.arange(start, start + n, dtype=torch.int32, device=device)[:, None].expand(n, bs)
        quantize_kv_paged(k, v, kv, blocks, offsets[None].expand(n, bs))


def empty_pool(kind: str, num_blocks: int, block_size: int, kv_heads: int, head_dim: int, device, block_table,
               scale: float = FP8_SCALE) -> PagedQuantKV:
    shape = (num_blocks, block_size, kv_heads, head_dim)
    if kind == "fp8":
        return PagedQuantKV("fp8", torch.zeros(shape, dtype=torch.uint8, device=device),
                            torch.zeros(shape, dtype=torch.uint8, device=device), block_table, block_size, scale, scale)
    if kind == "int8":
        sshape = shape[:3]
        return PagedQuantKV("int8", torch.zeros(shape, dtype=torch.int8, device=device),
                            torch.zeros(shape, dtype=torch.int8, device=device), block_table, block_size,
                            torch.ones(sshape, dtype=torch.float16, device=device),
                            torch.ones(sshape, dtype=torch.float16, device=device))
    raise ValueError(f"kind must be 'fp8' or 'int8', got {kind!r}")


def paged_case(kind: str = "fp8", batch: int = 32, q_heads: int = 16, kv_heads: int = 8, head_dim: int = 128,
               lengths: tuple[int, int] | list[int] = (512, 4096), block_size: int = 16, num_blocks: int = 16384,
               seed: int = 0, device="cuda", table_width: int | None = None,
               lengths_seed: int | None = None) -> PagedCase:
    """A filled paged pool, a random block table, ragged lengths and bf16 queries.

    `lengths` is either an inclusive range (lo, hi) drawn uniformly per sequence or an explicit list. A range is drawn
    with `lengths_seed` when it is given and differs from `seed` (the same lengths for batches whose content differs,
    e.g. one per rank of a weak-scaling run), else from the case's own generator first.
    """
    g = torch.Generator().manual_seed(seed)
    lg = g if lengths_seed is None or lengths_seed == seed else torch.Generator().manual_seed(lengths_seed)
    if isinstance(lengths, tuple):
        lo, hi = lengths
        lens = torch.randint(lo, hi + 1, (batch,), generator=lg, dtype=torch.int64)
    else:
        lens = torch.tensor(lengths, dtype=torch.int64)
    table = block_table_for(lens, block_size, num_blocks, g, table_width)
    q = torch.randn(batch, q_heads, head_dim, generator=g).to(torch.bfloat16)
    kv = empty_pool(kind, num_blocks, block_size, kv_heads, head_dim, device, table.to(device))
    fill_pool(kv, seed + 1)
    return PagedCase(q.to(device), kv, lens.to(torch.int32).to(device), q_heads)


def config1(device="cuda", seed: int = 0, keep_dense: bool = False) -> W4A16Case:
    return w4a16_case(1, 6144, 2048, 128, seed, device, keep_dense)


def config2(device="cuda", seed: int = 0, lengths_seed: int | None = None) -> PagedCase:
    return paged_case("fp8", 32, 16, 8, 128, (512, 4096), 16, 16384, seed, device, lengths_seed=lengths_seed)


def config3(device="cuda", seed: int = 0) -> PagedCase:
    return paged_case("int8", 8, 16, 8, 128, [32768] * 8, 16, 16384, seed, device)
