"""The quantized KV-cache write path on sm_100a.

- `quantize_kv_paged(k, v, kv, write_blocks, write_offsets)`: quantize this step's keys and values
  [B, Hkv, Q, D] to FP8 or INT8 and scatter them into a `PagedQuantKV` pool. The write of
  `PagedKVCache.update` (`src/fastserve/engine/kv_cache.py:150-161`) with the store of `kv/quant.py:40-48`
  in front of it.
- `quantize_kv(k, v, bits, group)`: the reference's `kernels/reference.py:132-160` (KIVI codes and grids) on
  the GPU, returning a `QuantKV`; `quantize_kv_into` writes whole groups into an existing cache, as
  `QuantizedKVCache._append` does (`integration/kv_cache.py:139-158`).
"""

from __future__ import annotations

import torch

from bpt_b200 import _lib
from bpt_b200._lib import check, dtype_code, lib, ptr, require_cuda, stream_of
from bpt_b200.kernels.kv_attention import PagedQuantKV, QuantKV


def quantize_kv_paged(k: torch.Tensor, v: torch.Tensor, kv: PagedQuantKV, write_blocks: torch.Tensor,
                      write_offsets: torch.Tensor) -> None:
    """Store k, v [B, Hkv, Q, D] at slot write_offsets[b, i] of block write_blocks[b, i] (int32 [B, Q])."""
    device = require_cuda(k, v, kv.k_pool, write_blocks, write_offsets)
    if k.shape != v.shape or k.dim() != 4:
        raise ValueError(f"k and v must both be [B, Hkv, Q, D], got {tuple(k.shape)} and {tuple(v.shape)}")
    if k.stride() != v.stride() or k.stride(-1) != 1:
        k, v = k.contiguous(), v.contiguous()
    b, hkv, q, d = k.shape
    nb, bs, hkv_pool, d_pool = kv.k_pool.shape
    if (hkv, d) != (hkv_pool, d_pool):
        raise ValueError(f"k has {hkv} heads of {d}, the pool {hkv_pool} of {d_pool}")
    wb = write_blocks.to(torch.int32).contiguous()
    wo = write_offsets.to(torch.int32).contiguous()
    if tuple(wb.shape) != (b, q) or tuple(wo.shape) != (b, q):
        raise ValueError(f"write_blocks / write_offsets must be [{b}, {q}]")
    if kv.kind == "fp8":
        code, ks, vs, kss, vss = _lib.KV_FP8, float(kv.k_scale), float(kv.v_scale), None, None
    elif kv.kind == "int8":
        code, ks, vs, kss, vss = _lib.KV_INT8, 1.0, 1.0, kv.k_scale, kv.v_scale
    else:
        raise ValueError(f"kind must be 'fp8' or 'int8', got {kv.kind!r}")
    st = lib().bpt_paged_kv_write(
        ptr(k), ptr(v), dtype_code(k.dtype), k.stride(0), k.stride(1), k.stride(2), b, hkv, q, d, ptr(wb), ptr(wo),
        ptr(kv.k_pool), ptr(kv.v_pool), code, ks, vs, ptr(kss), ptr(vss), bs, nb, stream_of(device))
    check(st, "quantize_kv_paged")


def empty_quant_kv(batch: int, kv_heads: int, tokens: int, head_dim: int, bits: int, group: int, device,
                   dtype=torch.bfloat16) -> QuantKV:
    """A zeroed KIVI cache laid out as QuantizedKVCache allocates one (integration/kv_cache.py:84-107)."""
    if bits == 16:
        shape = (batch, kv_heads, tokens, head_dim)
        return QuantKV(16, group, torch.zeros(shape, dtype=dtype, device=device), torch.zeros(shape, dtype=dtype, device=device))
    codes = (batch, kv_heads, tokens, head_dim // 2 if bits == 4 else head_dim)

    def grid(*shape):
        return torch.zeros(shape, dtype=torch.float16, device=device)

    return QuantKV(bits, group, torch.zeros(codes, dtype=torch.uint8, device=device),
                   torch.zeros(codes, dtype=torch.uint8, device=device), grid(batch, kv_heads, tokens // group, head_dim),
                   grid(batch, kv_heads, tokens // group, head_dim), grid(batch, kv_heads, tokens),
                   grid(batch, kv_heads, tokens))


def quantize_kv_into(k: torch.Tensor, v: torch.Tensor, kv: QuantKV, t0: int) -> None:
    """Quantize whole key groups k, v [B, Hkv, T, D] into `kv` at token offset t0 (a group boundary)."""
    device = require_cuda(k, v, kv.k_codes)
    if kv.bits == 16:
        kv.k_codes[:, :, t0 : t0 + k.shape[2]] = k
        kv.v_codes[:, :, t0 : t0 + v.shape[2]] = v
        return
    b, h, t, d = k.shape
    if t % kv.group:
        raise ValueError(f"{t} tokens are not a whole number of groups of {kv.group}")
    k, v = k.contiguous(), v.contiguous()
    st = lib().bpt_kivi_quantize(
        ptr(k), ptr(v), dtype_code(k.dtype), b, h, t, d, kv.bits, kv.group, ptr(kv.k_codes), ptr(kv.v_codes),
        ptr(kv.k_scale), ptr(kv.k_zero), ptr(kv.v_scale), ptr(kv.v_zero), kv.k_codes.shape[2], kv.k_scale.shape[2], t0,
        stream_of(device))
    check(st, "quantize_kv")


def quantize_kv(k: torch.Tensor, v: torch.Tensor, bits: int, group: int = 32) -> QuantKV:
    """reference.quantize_kv on the GPU: k, v [B, Hkv, T, D] -> a QuantKV holding exactly T tokens."""
    if bits == 16:
        return QuantKV(16, group, k.contiguous(), v.contiguous())
    if bits not in (4, 8):
        raise ValueError(f"bits must be 4, 8 or 16, got {bits}")
    b, h, t, d = k.shape
    if t % group:
        raise ValueError(f"{t} tokens are not a whole number of groups of {group}")
    kv = empty_quant_kv(b, h, t, d, bits, group, k.device)
    quantize_kv_into(k, v, kv, 0)
    return kv
