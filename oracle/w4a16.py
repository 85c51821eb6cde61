"""Oracle: asymmetric INT4 group-wise weight-only linear (W4A16), restated on the CPU. TEST INFRASTRUCTURE ONLY.

The reference has no W4A16 kernel. Its arithmetic for this path is spread over three places, which this file
restates in one:

- the asymmetric grid and the codes: `src/fastserve/quant/rtn.py:77-92` (`scale_and_zero`, asymmetric branch)
  and `:107-114` (`quantize`), with groups along the input dimension (`grouped`, `:65-74`);
- the storage layout: `src/fastserve/quant/compressed.py:25-53` (`pack_int` / `unpack_int`): eight 4-bit
  values per int32 word, value i of a row at bits 4i..4i+3 of word i/8;
- dequantize then matmul: `rtn.py:103-104` (`(q - zero) * scale`) and `compressed.py:56-69`
  (`dequantize_linear`), followed by `nn.Linear` (`src/fastserve/engine/model.py:43-46`).

Stored format (the one the CUDA kernels read):

    qweight  int32 [N, K/8]        code k of row n at bits 4(k mod 8) of word k/8, UNSIGNED 0..15 (no +8)
    scales   fp16  [N, K/group]    (max - min) / 15 of the group, range stretched to include 0
    qzeros   int32 [N, ceil(G/8)]  zero-point g of row n at bits 4(g mod 8) of word g/8, unsigned 0..15

Two deliberate, documented differences from `rtn.quantize`:

1. The scale is rounded to fp16 *before* the codes are computed (the convention of
   `src/fastserve/kernels/reference.py:103-114`, `_grid`), so codes and stored scale agree exactly.
   `rtn_quantize_asym` below restates rtn.quantize itself (fp32 scale) and is pinned by the golden vectors.
2. An all-zero group gets scale 1.0 (as `_grid`), since fp16 cannot hold rtn's 1e-12 floor.

Packing unsigned codes u is `pack_int(u - 8)` of compressed-tensors (which adds 8 back): the golden vectors pin
that identity. With no zero-points the format is compressed-tensors' symmetric pack-quantized layout, read
with an implicit zero-point of 8 (`compressed.py:1-15`).
"""

from __future__ import annotations

import torch


def grouped(w: torch.Tensor, group: int) -> torch.Tensor:
    """W [rows, cols] viewed as [rows, cols/group, group]. Follows rtn.py:65-74 (granularity "group")."""
    rows, cols = w.shape
    if cols % group:
        raise ValueError(f"{cols} input features are not divisible by group size {group}")
    return w.reshape(rows, cols // group, group)


def rtn_scale_and_zero_asym(x: torch.Tensor, bits: int) -> tuple[torch.Tensor, torch.Tensor]:
    """rtn.scale_and_zero, asymmetric branch (rtn.py:86-92): the grid over the last dim, fp32, [..., 1]."""
    x = x.float()
    lo = x.amin(dim=-1, keepdim=True).clamp(max=0)
    hi = x.amax(dim=-1, keepdim=True).clamp(min=0)
    scale = (hi - lo) / (2**bits - 1)
    zero = torch.round(-lo / scale.clamp(min=1e-12))
    return scale.clamp(min=1e-12), zero


def rtn_quantize_asym(w: torch.Tensor, bits: int = 4, group: int = 128):
    """rtn.quantize with IntSpec(bits, "group", group, symmetric=False) (rtn.py:107-114).

    Returns (q [rows, n_groups, group] float, scale [rows, n_groups, 1], zero [rows, n_groups, 1]).
    """
    x = grouped(w.float(), group)
    scale, zero = rtn_scale_and_zero_asym(x, bits)
    return torch.clamp(torch.round(x / scale) + zero, 0, 2**bits - 1), scale, zero


def quantize_w4a16(w: torch.Tensor, group: int = 128) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The stored W4A16 grid: (codes uint8 [N, K] in 0..15, scales fp16 [N, G], zeros uint8 [N, G]).

    rtn.py:86-92 and :113-114 with the fp16-scale-first convention of reference.py:109-114.
    """
    x = grouped(w.float(), group)  # [N, G, group]
    lo = x.amin(dim=-1, keepdim=True).clamp(max=0)
    hi = x.amax(dim=-1, keepdim=True).clamp(min=0)
    scale = ((hi - lo) / 15).to(torch.float16)
    scale = torch.where(scale > 0, scale, torch.ones_like(scale))
    zero = torch.round(-lo / scale.float()).clamp(0, 15)
    codes = torch.clamp(torch.round(x / scale.float()) + zero, 0, 15)
    n = w.shape[0]
    return (
        codes.reshape(n, -1).to(torch.uint8),
        scale.reshape(n, -1),
        zero.reshape(n, -1).to(torch.uint8),
    )


def pack_nibbles_int32(codes: torch.Tensor) -> torch.Tensor:
    """Unsigned 4-bit values [rows, cols] -> int32 words [rows, ceil(cols/8)], value i at bits 4(i mod 8).

    compressed.pack_int (compressed.py:25-41) without its +8 offset: the values are already unsigned.
    A row that does not fill its last word is padded with zero bits.
    """
    rows, cols = codes.shape
    u = codes.to(torch.int64) & 0xF
    u = torch.nn.functional.pad(u, (0, -cols % 8)).reshape(rows, -1, 8)
    shifts = torch.arange(8, dtype=torch.int64) * 4
    words = (u << shifts).sum(dim=-1)
    return torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)


def unpack_nibbles_int32(packed: torch.Tensor, cols: int) -> torch.Tensor:
    """Inverse of `pack_nibbles_int32`: int32 [rows, words] -> uint8 [rows, cols] (compressed.py:44-53)."""
    shifts = torch.arange(8, dtype=torch.int32) * 4
    fields = (packed.unsqueeze(-1) >> shifts) & 0xF
    return fields.reshape(packed.shape[0], -1)[:, :cols].to(torch.uint8)


def dequantize_w4a16(codes: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, group: int) -> torch.Tensor:
    """Dense fp32 weight [N, K] = scale * (code - zero) per group (rtn.py:103-104; compressed.py:56-69).

    zeros None: compressed-tensors' symmetric layout, an implicit zero-point of 8 (compressed.py:28-31).
    """
    q = codes.float()
    z = torch.full_like(scales, 8, dtype=torch.float32) if zeros is None else zeros.float()
    s = scales.float()
    return (q - z.repeat_interleave(group, dim=1)) * s.repeat_interleave(group, dim=1)


def w4a16_linear(
    x: torch.Tensor,
    qweight: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor | None,
    group: int = 128,
    bias: torch.Tensor | None = None,
    dense_bf16: bool = False,
) -> torch.Tensor:
    """y = x @ W^T in fp32 from the packed format, returned in x's dtype.

    The reference path: unpack (compressed.py:44-53), dequantize (rtn.py:103-104), then a float32
    `F.linear` (engine/model.py:43-46 runs nn.Linear), rounded once to the activation dtype.
    dense_bf16: the weight the reference's model actually holds, `dequantize_linear` (compressed.py:56-69):
    each product s (q - z), exact in float32, rounded once to bf16, then the fp32-accumulated matmul.
    """
    n, k = qweight.shape[0], qweight.shape[1] * 8
    codes = unpack_nibbles_int32(qweight, k)
    zeros = None if qzeros is None else unpack_nibbles_int32(qzeros, k // group)
    w = dequantize_w4a16(codes, scales, zeros, group)
    if dense_bf16:
        w = w.to(torch.bfloat16).float()
    y = torch.nn.functional.linear(x.float(), w, None if bias is None else bias.float())
    return y.to(x.dtype)


def w4a16_gate_up_silu(
    x: torch.Tensor,
    qweight: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor | None,
    group: int = 128,
    dense_bf16: bool = False,
) -> torch.Tensor:
    """silu(g) * u for a fused gate/up weight whose rows alternate gate (2i) and up (2i + 1), in x's dtype.

    The MLP of `src/fastserve/engine/model.py:95-96` (`down(silu(gate(x)) * up(x))`) up to its input of down_proj,
    with g and u kept in fp32 from the fp32-accumulated matmul (`w4a16_linear` above, before its final rounding)
    and one rounding at the end: the arithmetic that fp32 accumulation prescribes. The reference model rounds g
    and u to bf16 first (its nn.Linear outputs); that rounding is left out here on purpose.
    """
    n, k = qweight.shape[0], qweight.shape[1] * 8
    codes = unpack_nibbles_int32(qweight, k)
    zeros = None if qzeros is None else unpack_nibbles_int32(qzeros, k // group)
    w = dequantize_w4a16(codes, scales, zeros, group)
    if dense_bf16:
        w = w.to(torch.bfloat16).float()
    y = torch.nn.functional.linear(x.float(), w)
    g, u = y[..., 0::2], y[..., 1::2]
    return (torch.nn.functional.silu(g) * u).to(x.dtype)


def pack_w4a16(codes: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor):
    """(codes, scales, zeros) -> the stored tensors (qweight, scales, qzeros)."""
    return pack_nibbles_int32(codes), scales.contiguous(), pack_nibbles_int32(zeros)
