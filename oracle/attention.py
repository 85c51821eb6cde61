"""Oracle: decode attention over a quantized cache, the unfused way, on the CPU. TEST INFRASTRUCTURE ONLY.

- `partial_attention` / `merge_partials`: `src/fastserve/kernels/reference.py:186-211`, with GQA by
  `repeat_kv` (`src/fastserve/engine/attention.py:23-31`: KV head h serves query heads h*REP ... h*REP+REP-1).
- `paged_gather`: `PagedKVCache._gather` (`src/fastserve/engine/kv_cache.py:165-169`).
- `paged_decode_partials`: gather, dequantize (`oracle.kv_formats`), then one `partial_attention` per split of
  `split` tokens: the per-split (out, lse) contract of kernel 2 (`src/fastserve/kernels/kv_attention.py:
  167-173`): a split past a row's end has out 0 and lse -inf.
- `kivi_decode_attention`: `reference.decode_attention` (`reference.py:214-224`).
"""

from __future__ import annotations

import torch

from oracle.kv_formats import KiviKV, PagedKV, fp8_load, int8_load, kivi_dequantize


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """[B, Hkv, T, D] -> [B, Hkv * n_rep, T, D] (engine/attention.py:23-31)."""
    if n_rep == 1:
        return x
    b, h, t, d = x.shape
    return x[:, :, None].expand(b, h, n_rep, t, d).reshape(b, h * n_rep, t, d)


def partial_attention(q, k, v, lengths, scale):
    """(out [B, Hq, D], lse [B, Hq]) of one query per head over k, v [B, Hkv, T, D] (reference.py:186-202)."""
    group = q.shape[1] // k.shape[1]
    k, v = repeat_kv(k.float(), group), repeat_kv(v.float(), group)
    scores = torch.einsum("bhd,bhtd->bht", q.float(), k) * scale
    visible = torch.arange(k.shape[2])[None, :] < lengths.to(torch.int64)[:, None]
    scores = scores.masked_fill(~visible[:, None], float("-inf"))
    lse = torch.logsumexp(scores, dim=-1)
    probs = torch.softmax(scores, dim=-1).nan_to_num(0.0)
    return torch.einsum("bht,bhtd->bhd", probs, v), lse


def merge_partials(outs: torch.Tensor, lses: torch.Tensor) -> torch.Tensor:
    """[B, Hq, S, D], [B, Hq, S] -> [B, Hq, D] (reference.py:205-211)."""
    share = torch.softmax(lses, dim=-1).nan_to_num(0.0)
    return (share[..., None] * outs).sum(dim=2)


def paged_gather(pool: torch.Tensor, block_table: torch.Tensor, kv_len: int) -> torch.Tensor:
    """pool [num_blocks, block_size, Hkv, ...] -> [B, Hkv, kv_len, ...] (engine/kv_cache.py:165-169)."""
    b, n = block_table.shape
    bs = pool.shape[1]
    blocks = pool[block_table.to(torch.int64)]  # [B, n, bs, Hkv, ...]
    flat = blocks.reshape(b, n * bs, *pool.shape[2:])[:, :kv_len]
    return flat.transpose(1, 2)


def paged_dequantize(kv: PagedKV, kv_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Every sequence's first kv_len keys and values, gathered and dequantized: fp32 [B, Hkv, kv_len, D]."""
    k_codes = paged_gather(kv.k_pool, kv.block_table, kv_len)
    v_codes = paged_gather(kv.v_pool, kv.block_table, kv_len)
    if kv.kind == "fp8":
        return fp8_load(k_codes, float(kv.k_scale)), fp8_load(v_codes, float(kv.v_scale))
    k_scale = paged_gather(kv.k_scale[..., None], kv.block_table, kv_len)[..., 0]  # [B, Hkv, kv_len]
    v_scale = paged_gather(kv.v_scale[..., None], kv.block_table, kv_len)[..., 0]
    return int8_load(k_codes, k_scale), int8_load(v_codes, v_scale)


def paged_decode_partials(q, kv: PagedKV, lengths, scale: float, split: int, tokens: int | None = None):
    """Per-split partial attentions over a paged quantized cache: (out [B, Hq, S, D], lse [B, Hq, S]).

    S = ceil(tokens / split), at least 1; `tokens` defaults to max(lengths).
    """
    lengths = lengths.to(torch.int64)
    tokens = int(lengths.max()) if tokens is None else tokens
    n_splits = max(-(-tokens // split), 1)
    kv_len = n_splits * split
    max_len = kv.block_table.shape[1] * kv.block_size
    kv_len_g = min(kv_len, max_len)
    k, v = paged_dequantize(kv, kv_len_g)
    outs, lses = [], []
    for s in range(n_splits):
        start = s * split
        seen = (lengths - start).clamp(0, split)
        out, lse = partial_attention(q, k[:, :, start : start + split], v[:, :, start : start + split], seen, scale)
        outs.append(out)
        lses.append(lse)
    return torch.stack(outs, dim=2), torch.stack(lses, dim=2)


def paged_attend(q, kv: PagedKV, lengths, scale: float) -> torch.Tensor:
    """Decode attention over a paged quantized cache in one piece: [B, Hq, D] fp32."""
    lengths = lengths.to(torch.int64)
    kv_len = max(int(lengths.max()), 1)
    k, v = paged_dequantize(kv, kv_len)
    out, _ = partial_attention(q, k, v, lengths, scale)
    return out


def kivi_decode_attention(q, kv: KiviKV, lengths, scale: float):
    """reference.decode_attention (reference.py:214-224): (out [B, Hq, 1, D], lse [B, Hq, 1])."""
    k, v = kivi_dequantize(kv)
    out, lse = partial_attention(q, k, v, lengths, scale)
    return out[:, :, None], lse[:, :, None]
