"""The decode step's small ops around the hot path, fused (config 5's caller side; `csrc/decode_fused.cu`).

`rms_norm_residual` is RMSNorm (`engine/model.py:24-36`) with the residual add of `DecoderLayer.forward`
(`:109-111`) in front; `qk_norm_rope_kv_write` is the q_norm / k_norm, rotary embedding and cache write of
`Attention.forward` (`:63-70`, `engine/rope.py:31-43`, `engine/kv_cache.py:150-161`) for one new token per
sequence into an FP8 paged cache. Both keep every bf16 rounding of the reference's tensors.
"""

from __future__ import annotations

import torch

from bpt_b200._lib import FLAG_PDL, check, lib, ptr, require_cuda, stream_of
from bpt_b200.kernels.kv_attention import PagedQuantKV


def rms_norm_residual(h: torch.Tensor, weight: torch.Tensor, eps: float, *, delta: torch.Tensor | None = None,
                      h_out: torch.Tensor | None = None, x_out: torch.Tensor | None = None, pdl: bool = False):
    """(h + delta or h, RMSNorm of it) for bf16 [rows, hidden]; the sum goes to h_out (if given), the norm to x."""
    device = require_cuda(h, weight, delta, h_out, x_out)
    if h.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or h.dim() != 2 or not h.is_contiguous():
        raise ValueError("rms_norm_residual takes contiguous bf16 h [rows, hidden] and a bf16 weight")
    rows, hidden = h.shape
    for t in (delta, h_out, x_out):
        if t is not None and (t.shape != h.shape or t.dtype != h.dtype or not t.is_contiguous()):
            raise ValueError("delta, h_out and x_out must match h")
    if weight.shape != (hidden,):
        raise ValueError(f"weight must be [{hidden}]")
    x = x_out if x_out is not None else torch.empty_like(h)
    st = lib().bpt_rms_norm_residual(ptr(h), ptr(delta), ptr(weight), ptr(h_out), ptr(x), rows, hidden, float(eps),
                                     FLAG_PDL if pdl else 0, stream_of(device))
    check(st, "rms_norm_residual")
    return h_out, x


def qk_norm_rope_kv_write(qkv: torch.Tensor, q_heads: int, kv_heads: int, q_norm: torch.Tensor,
                          k_norm: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, eps: float, kv: PagedQuantKV,
                          write_blocks: torch.Tensor, write_offsets: torch.Tensor, *, q_out: torch.Tensor,
                          pdl: bool = False) -> torch.Tensor:
    """qkv [B, (Hq + 2 Hkv) * 128] bf16 -> q_out [B, Hq, 128] (normed, rotated); k and v stored in the FP8 pools."""
    device = require_cuda(qkv, q_norm, k_norm, cos, sin, kv.k_pool, write_blocks, write_offsets, q_out)
    if kv.kind != "fp8":
        raise ValueError("qk_norm_rope_kv_write stores into an FP8 cache")
    b = qkv.shape[0]
    d = 128
    if qkv.dim() != 2 or qkv.stride(1) != 1 or qkv.shape[1] < (q_heads + 2 * kv_heads) * d:
        raise ValueError("qkv must be [B, (Hq + 2 Hkv) * 128] with unit inner stride")
    if tuple(q_out.shape) != (b, q_heads, d) or not q_out.is_contiguous():
        raise ValueError(f"q_out must be a contiguous [{b}, {q_heads}, {d}] tensor")
    wb = write_blocks.reshape(b).to(torch.int32).contiguous()
    wo = write_offsets.reshape(b).to(torch.int32).contiguous()
    nb, bs = kv.k_pool.shape[0], kv.k_pool.shape[1]
    st = lib().bpt_qk_norm_rope_kv_write(
        ptr(qkv), qkv.stride(0), b, q_heads, kv_heads, d, ptr(q_norm), ptr(k_norm), ptr(cos.contiguous()),
        ptr(sin.contiguous()), float(eps), ptr(q_out), ptr(wb), ptr(wo), ptr(kv.k_pool), ptr(kv.v_pool),
        float(kv.k_scale), float(kv.v_scale), bs, nb, FLAG_PDL if pdl else 0, stream_of(device))
    check(st, "qk_norm_rope_kv_write")
    return q_out
