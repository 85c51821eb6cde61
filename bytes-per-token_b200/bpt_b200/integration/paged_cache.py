"""A paged KV cache for nanoserve that stores FP8 or INT8 codes and attends over them with this package's kernels.

The reference has two caches that meet at this seam:

- `PagedKVCache` (`src/fastserve/engine/kv_cache.py:98-169`): a pool of fixed-size blocks with a block table per
  sequence, host-side block management (`reserve` / `free`), and a bf16 read that gathers every page back into a
  contiguous tensor (`_gather`, `:165-169`) before attention;
- `QuantizedKVCache` (`src/fastserve/integration/kv_cache.py:59-192`): a cache that stores codes and exposes
  `attend(layer, q, k, v, meta, scale)`, which `Attention.forward` calls instead of `update` when the cache has
  it (`engine/model.py:72-74`); its decode read is an injected `DecodeFn` (`:38-39`) whose per-split partials
  `merge_partials` joins.

`PagedQuantizedKVCache` is the paged cache with the quantized cache's `attend` seam, so nanoserve's model drives
it unchanged:

- **write** (`_append`): this step's k, v [B, Hkv, Q, D] are quantized and scattered to their (block, slot) by one
  `quantize_kv_paged` launch (FP8 E4M3 with a per-tensor scale, or symmetric INT8 with an fp16 scale per token and
  KV head). There is no full-precision tail: every token is quantized on its own, so none waits for a group.
- **decode read** (one new token per row): the paged decode attention reads the codes straight from the pages
  through the block table. By default one fused launch (`kv_attention.attend`: split-K with the merge in the same
  kernel); with `decode=` a `DecodeFn` such as `kv_attention.decode_attention` returns per-split partials that
  `merge_partials` joins, as the reference's cache does.
- **prefill read** (several new tokens): the unfused path, as in the reference (`integration/kv_cache.py:187-192`):
  the pages are gathered and dequantized, then a causal GQA attention runs in PyTorch. The decode kernel is a
  decode kernel; prefill is compute-bound and not where the cache's bytes matter.

Every tensor lives on one CUDA device; there is no CPU path.
"""

from __future__ import annotations

import dataclasses
import math
from collections.abc import Callable
from dataclasses import dataclass
from typing import Any

import torch

from bpt_b200._lib import require_cuda
from bpt_b200.kernels.kv_attention import PagedQuantKV, attend, merge_partials
from bpt_b200.kernels.kv_write import quantize_kv_paged

# (q [B, Hq, D], kv, lengths [B], scale, tokens) -> (out [B, Hq, S, D], lse [B, Hq, S]), integration/kv_cache.py:38-39
DecodeFn = Callable[..., tuple[torch.Tensor, torch.Tensor]]


class OutOfBlocksError(RuntimeError):
    """The pool has no free block (engine/kv_cache.py:86-87): the scheduler must wait or preempt a sequence."""


@dataclass(frozen=True)
class PagedQuantMeta:
    """Per-forward metadata, computed once by `prepare` and shared by every layer (engine/kv_cache.py:90-95)."""

    positions: torch.Tensor  # [B, Q] absolute positions of the new tokens
    write_blocks: torch.Tensor  # int32 [B, Q] physical block receiving each new token
    write_offsets: torch.Tensor  # int32 [B, Q] slot inside that block
    block_table: torch.Tensor  # int32 [B, n_blocks] physical blocks of logical blocks 0 .. n_blocks - 1
    lengths: torch.Tensor  # int32 [B] tokens each row attends over once this write is in (last position + 1)
    kv_len: int  # the longest row's length
    q_len: int


class PagedQuantizedKVCache:
    """Paged FP8 / INT8 KV cache with the `attend` seam of the reference's quantized cache.

    cfg: anything with `num_layers`, `num_kv_heads` and `head_dim` (the reference's `ModelConfig`,
    `engine/config.py:15-27`). kind "fp8": `k_scale` / `v_scale` are the per-tensor scales (x / scale is stored);
    kind "int8": the scales are per (token, KV head) and computed on write.
    """

    def __init__(self, cfg: Any, *, num_blocks: int, block_size: int = 16, kind: str = "fp8",
                 k_scale: float = 1.0, v_scale: float = 1.0, device: torch.device | str = "cuda",
                 decode: DecodeFn | None = None):
        if kind not in ("fp8", "int8"):
            raise ValueError(f"kind must be 'fp8' or 'int8', got {kind!r}")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("PagedQuantizedKVCache lives on a CUDA device: its kernels have no CPU path")
        self.kind, self.block_size, self.num_blocks, self.decode = kind, block_size, num_blocks, decode
        shape = (num_blocks, block_size, cfg.num_kv_heads, cfg.head_dim)  # engine/kv_cache.py:108
        empty_table = torch.zeros(0, 1, dtype=torch.int32, device=self.device)

        def layer() -> PagedQuantKV:
            if kind == "fp8":
                return PagedQuantKV("fp8", torch.zeros(shape, dtype=torch.uint8, device=self.device),
                                    torch.zeros(shape, dtype=torch.uint8, device=self.device), empty_table, block_size,
                                    float(k_scale), float(v_scale))
            return PagedQuantKV("int8", torch.zeros(shape, dtype=torch.int8, device=self.device),
                                torch.zeros(shape, dtype=torch.int8, device=self.device), empty_table, block_size,
                                torch.ones(shape[:3], dtype=torch.float16, device=self.device),
                                torch.ones(shape[:3], dtype=torch.float16, device=self.device))

        self.layers = [layer() for _ in range(cfg.num_layers)]
        self.free_blocks = list(range(num_blocks - 1, -1, -1))  # a stack: pop() hands out block 0 first
        self.tables: dict[Any, list[int]] = {}  # sequence id -> its block table

    # -- memory management (host side, engine/kv_cache.py:117-138) --------------------------------------------------

    def blocks_needed(self, num_tokens: int) -> int:
        return math.ceil(num_tokens / self.block_size)

    def can_reserve(self, seq_id: Any, num_tokens: int) -> bool:
        have = len(self.tables.get(seq_id, []))
        return self.blocks_needed(num_tokens) - have <= len(self.free_blocks)

    def reserve(self, seq_id: Any, num_tokens: int) -> None:
        """Make sure `seq_id` owns enough blocks to hold positions [0, num_tokens)."""
        table = self.tables.setdefault(seq_id, [])
        missing = self.blocks_needed(num_tokens) - len(table)
        if missing > len(self.free_blocks):
            raise OutOfBlocksError(f"need {missing} blocks, {len(self.free_blocks)} free")
        table.extend(self.free_blocks.pop() for _ in range(missing))

    def free(self, seq_id: Any) -> None:
        """Return a finished sequence's blocks to the pool."""
        self.free_blocks.extend(reversed(self.tables.pop(seq_id, [])))

    def bytes_per_token(self) -> float:
        """Bytes one token occupies across all layers and KV heads, scales included."""
        return sum(kv.bytes_per_token() for kv in self.layers)

    # -- the KVCache interface ------------------------------------------------------------------------------------

    def prepare(self, rows: list[Any], positions: torch.Tensor) -> PagedQuantMeta:
        """Write slots and block table for this forward (engine/kv_cache.py:140-156), plus each row's length.

        Rows may sit at different positions (continuous batching); each attends over its own last position + 1.
        """
        positions = positions.to(self.device)
        b, q_len = positions.shape
        if len(rows) != b:
            raise ValueError(f"{len(rows)} rows for a batch of {b}")
        last = positions.max(dim=1).values.cpu().tolist()
        kv_len = int(max(last)) + 1
        n_blocks = self.blocks_needed(kv_len)
        tables = []
        for i, seq_id in enumerate(rows):
            table = self.tables[seq_id]
            if len(table) * self.block_size < int(last[i]) + 1:
                raise ValueError(f"sequence {seq_id!r} has too few blocks: call reserve() first")
            tables.append(table[:n_blocks] + [0] * (n_blocks - len(table)))  # padded entries are never read
        block_table = torch.tensor(tables, dtype=torch.int32).to(self.device)
        logical = (positions // self.block_size).to(torch.int64)
        return PagedQuantMeta(
            positions=positions,
            write_blocks=torch.gather(block_table, 1, logical).to(torch.int32),
            write_offsets=(positions % self.block_size).to(torch.int32),
            block_table=block_table,
            lengths=torch.tensor([int(p) + 1 for p in last], dtype=torch.int32).to(self.device),
            kv_len=kv_len,
            q_len=q_len,
        )

    def update(self, layer: int, k: torch.Tensor, v: torch.Tensor, meta: PagedQuantMeta):
        raise NotImplementedError("a quantized cache never returns float keys and values: use attend()")

    def _append(self, layer: int, k: torch.Tensor, v: torch.Tensor, meta: PagedQuantMeta) -> None:
        """Quantize k, v [B, Hkv, Q, D] into the layer's pools at the metadata's slots (one launch)."""
        quantize_kv_paged(k, v, self.layers[layer], meta.write_blocks, meta.write_offsets)

    def layer_view(self, layer: int, meta: PagedQuantMeta) -> PagedQuantKV:
        """The layer's pools with this forward's block table: what the attention kernels read."""
        return dataclasses.replace(self.layers[layer], block_table=meta.block_table)

    def attend(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, meta: PagedQuantMeta,
               scale: float) -> torch.Tensor:
        """Store this step's k, v, then attend: q [B, Hq, Q, D] -> [B, Hq, Q, D] in q's dtype.

        New tokens are stored before attention, so a query sees its own token as the cache holds it (the order of
        integration/kv_cache.py:160-170).
        """
        require_cuda(q, k, v)
        self._append(layer, k, v, meta)
        kv = self.layer_view(layer, meta)
        if meta.q_len == 1:  # decode: the paged kernel over the codes
            query = q[:, :, 0]
            if self.decode is None:
                return attend(query, kv, meta.lengths, scale, tokens=meta.kv_len)[:, :, None].to(q.dtype)
            out, lse = self.decode(query, kv, meta.lengths, scale, tokens=meta.kv_len)
            return merge_partials(out, lse)[:, :, None].to(q.dtype)
        # prefill: the unfused path (gather, dequantize, causal GQA attention)
        keys, values = self.dequantized(layer, meta)
        slots = torch.arange(meta.kv_len, device=q.device)
        mask = (slots[None, None, :] <= meta.positions[:, :, None])[:, None]  # engine/attention.py:12-20
        rep = q.shape[1] // keys.shape[1]
        keys = keys.to(q.dtype).repeat_interleave(rep, dim=1)
        values = values.to(q.dtype).repeat_interleave(rep, dim=1)
        return torch.nn.functional.scaled_dot_product_attention(q, keys, values, attn_mask=mask, scale=scale)

    def dequantized(self, layer: int, meta: PagedQuantMeta) -> tuple[torch.Tensor, torch.Tensor]:
        """Every row's first kv_len tokens, gathered through the block table and dequantized to fp32:
        [B, Hkv, kv_len, D] each (the read of engine/kv_cache.py:165-169 with the store's inverse)."""
        kv = self.layers[layer]
        b, n = meta.block_table.shape
        idx = meta.block_table.to(torch.int64)

        def gather(pool, scales):
            blocks = pool[idx]  # [B, n_blocks, block_size, Hkv, D]
            if kv.kind == "fp8":
                vals = blocks.view(torch.float8_e4m3fn).float() * float(scales)
            else:
                vals = blocks.float() * scales[idx].float()[..., None]
            flat = vals.reshape(b, n * self.block_size, *pool.shape[2:])[:, : meta.kv_len]
            return flat.transpose(1, 2)

        return gather(kv.k_pool, kv.k_scale), gather(kv.v_pool, kv.v_scale)
