"""Oracle: the quantized KV-cache formats, restated on the CPU. TEST INFRASTRUCTURE ONLY.

Three storage formats, each the reference's own arithmetic:

**FP8 E4M3, per-tensor scale.** `src/fastserve/kv/quant.py:44-45` stores `x.clamp(-448, 448)` cast to
`float8_e4m3fn` (scale 1.0, vLLM's default). The paged cache generalises the scale to any fp32 s:
code = e4m3(clamp(x / s, -448, 448)), read back as fp32(code) * s. Rounding is the cast's: nearest, ties to
even (pinned against the from-scratch rounding of `src/fastserve/quant/formats.py:43-52`).

**Symmetric INT8, one fp16 scale per (token, head).** `kv/quant.py:35-48` with axis "token" and group = head
dim runs `rtn.scale_and_zero` symmetric (`src/fastserve/quant/rtn.py:82-85`, qmax 127) and
`rtn.round_to_grid` (`rtn.py:100-102`): scale = absmax / 127, code = clamp(round(x / scale), -128, 127).
The stored scale is fp16, rounded *before* the codes (the `_grid` convention of
`src/fastserve/kernels/reference.py:103-114`), so codes and scale agree; an all-zero vector gets scale 1.0.
`int8_store_rtn` keeps rtn's fp32 scale and is pinned by the golden vectors.

**KIVI, contiguous** (`src/fastserve/kernels/reference.py:66-180`): asymmetric 4- or 8-bit grids, keys per
channel over groups of `group` tokens, values per token; 4-bit codes packed channel d low / d + D/2 high.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

FP8_MAX = 448.0  # kv/quant.py:30, the largest finite E4M3 value
INT8_MAX = 127.0


# ---- FP8 E4M3 ------------------------------------------------------------------------------------------------


def fp8_store(x: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """E4M3 codes of x / scale as uint8 bytes. kv/quant.py:44-45 with a general per-tensor scale."""
    y = (x.float() / scale).clamp(-FP8_MAX, FP8_MAX)
    return y.to(torch.float8_e4m3fn).view(torch.uint8)


def fp8_load(codes: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """fp32 values of E4M3 codes (uint8 bytes) times the per-tensor scale."""
    return codes.view(torch.float8_e4m3fn).float() * scale


# ---- symmetric INT8 per (token, head) ------------------------------------------------------------------------


def int8_store(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(codes int8 [..., D], scale fp16 [...]): one grid per vector along the last dim.

    rtn.py:82-85 (scale = max|x| / 127) and rtn.py:100-102 (clamp(round(x / s), -128, 127)), with the scale
    rounded to fp16 first and an all-zero vector given scale 1.0, as reference.py:111-112 does.
    """
    x32 = x.float()
    scale = (x32.abs().amax(dim=-1, keepdim=True) / INT8_MAX).to(torch.float16)
    scale = torch.where(scale > 0, scale, torch.ones_like(scale))
    codes = torch.clamp(torch.round(x32 / scale.float()), -128, 127).to(torch.int8)
    return codes, scale.squeeze(-1)


def int8_store_rtn(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """rtn's own symmetric INT8 over the last dim, fp32 scale (rtn.py:82-85, :111-113). Pinned by goldens."""
    x32 = x.float()
    scale = (x32.abs().amax(dim=-1, keepdim=True) / INT8_MAX).clamp(min=1e-12)
    codes = torch.clamp(torch.round(x32 / scale), -128, 127)
    return codes, scale


def int8_load(codes: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp32 values: code * scale, the scale broadcast over the last dim (rtn.py:102)."""
    return codes.float() * scale.float().unsqueeze(-1)


# ---- KIVI (contiguous) ---------------------------------------------------------------------------------------


@dataclass
class KiviKV:
    """The field names of reference.QuantKV (reference.py:66-86). Shapes as documented there."""

    bits: int
    group: int
    k_codes: torch.Tensor
    v_codes: torch.Tensor
    k_scale: torch.Tensor | None = None
    k_zero: torch.Tensor | None = None
    v_scale: torch.Tensor | None = None
    v_zero: torch.Tensor | None = None

    @property
    def tokens(self) -> int:
        return self.k_codes.shape[2]


def kivi_grid(x: torch.Tensor, bits: int, dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """reference._grid (reference.py:103-114): asymmetric grid along dim, fp16 scale and zero as stored."""
    lo = x.amin(dim, keepdim=True).clamp(max=0)
    hi = x.amax(dim, keepdim=True).clamp(min=0)
    scale = ((hi - lo) / (2**bits - 1)).to(torch.float16)
    scale = torch.where(scale > 0, scale, torch.ones_like(scale))
    zero = torch.round(-lo / scale.float()).clamp(0, 2**bits - 1).to(torch.float16)
    return scale, zero


def kivi_codes(x: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, bits: int) -> torch.Tensor:
    """reference._codes (reference.py:117-118)."""
    return torch.clamp(torch.round(x / scale.float()) + zero.float(), 0, 2**bits - 1).to(torch.uint8)


def pack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    """reference.pack_nibbles (reference.py:121-124): channel d low nibble, channel d + D/2 high nibble."""
    half = codes.shape[-1] // 2
    return codes[..., :half] | (codes[..., half:] << 4)


def unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    """reference.unpack_nibbles (reference.py:127-129)."""
    return torch.cat([packed & 0xF, packed >> 4], dim=-1)


def kivi_quantize(k: torch.Tensor, v: torch.Tensor, bits: int, group: int = 32) -> KiviKV:
    """reference.quantize_kv (reference.py:132-160): k, v [B, Hkv, T, D] -> stored codes and grids."""
    if bits == 16:
        return KiviKV(16, group, k.contiguous(), v.contiguous())
    b, h, t, d = k.shape
    if t % group:
        raise ValueError(f"{t} tokens are not a whole number of groups of {group}")
    k32, v32 = k.float(), v.float()
    blocks = k32.reshape(b, h, t // group, group, d)
    k_scale, k_zero = kivi_grid(blocks, bits, dim=3)
    k_codes = kivi_codes(blocks, k_scale, k_zero, bits).reshape(b, h, t, d)
    v_scale, v_zero = kivi_grid(v32, bits, dim=3)
    v_codes = kivi_codes(v32, v_scale, v_zero, bits)
    if bits == 4:
        k_codes, v_codes = pack_nibbles(k_codes), pack_nibbles(v_codes)
    return KiviKV(
        bits,
        group,
        k_codes.contiguous(),
        v_codes.contiguous(),
        k_scale.squeeze(3).contiguous(),
        k_zero.squeeze(3).contiguous(),
        v_scale.squeeze(3).contiguous(),
        v_zero.squeeze(3).contiguous(),
    )


def kivi_dequantize(kv: KiviKV, tokens: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """reference.dequantize_kv (reference.py:163-180): the first `tokens` keys and values in fp32."""
    t = kv.tokens if tokens is None else tokens
    if kv.bits == 16:
        return kv.k_codes[:, :, :t].float(), kv.v_codes[:, :, :t].float()
    k_codes, v_codes = kv.k_codes[:, :, :t], kv.v_codes[:, :, :t]
    if kv.bits == 4:
        k_codes, v_codes = unpack_nibbles(k_codes), unpack_nibbles(v_codes)
    groups = -(-t // kv.group)
    k_scale = kv.k_scale[:, :, :groups].float().repeat_interleave(kv.group, dim=2)[:, :, :t]
    k_zero = kv.k_zero[:, :, :groups].float().repeat_interleave(kv.group, dim=2)[:, :, :t]
    k = k_scale * (k_codes.float() - k_zero)
    v = kv.v_scale[:, :, :t, None].float() * (v_codes.float() - kv.v_zero[:, :, :t, None].float())
    return k, v


# ---- the paged pool --------------------------------------------------------------------------------------------


@dataclass
class PagedKV:
    """A paged, quantized pool for one layer, in the reference's paged layout (engine/kv_cache.py:108).

    k_pool, v_pool  [num_blocks, block_size, Hkv, D]  uint8 E4M3 bytes ("fp8") or int8 codes ("int8")
    k_scale/v_scale fp32 per-tensor scale ("fp8") or fp16 [num_blocks, block_size, Hkv] ("int8")
    block_table     int32 [B, max_blocks]: physical block of each sequence's logical block
    """

    kind: str
    k_pool: torch.Tensor
    v_pool: torch.Tensor
    k_scale: torch.Tensor | float
    v_scale: torch.Tensor | float
    block_table: torch.Tensor
    block_size: int


def store_vectors(x: torch.Tensor, kind: str, scale: float = 1.0):
    """Quantize vectors [..., D] in format `kind`: (codes, per-vector scales or None)."""
    if kind == "fp8":
        return fp8_store(x, scale), None
    if kind == "int8":
        return int8_store(x)
    raise ValueError(f"kind must be 'fp8' or 'int8', got {kind!r}")


def paged_write(kv: PagedKV, k: torch.Tensor, v: torch.Tensor, write_blocks: torch.Tensor, write_offsets: torch.Tensor):
    """Quantize k, v [B, Hkv, Q, D] and scatter token (b, i) to slot write_offsets[b, i] of block
    write_blocks[b, i]: PagedKVCache.update's write (engine/kv_cache.py:158-161) with the store in front."""
    kt, vt = k.transpose(1, 2), v.transpose(1, 2)  # [B, Q, Hkv, D]
    if kv.kind == "fp8":
        kv.k_pool[write_blocks, write_offsets] = fp8_store(kt, float(kv.k_scale))
        kv.v_pool[write_blocks, write_offsets] = fp8_store(vt, float(kv.v_scale))
    else:
        kc, ks = int8_store(kt)
        vc, vs = int8_store(vt)
        kv.k_pool[write_blocks, write_offsets] = kc
        kv.v_pool[write_blocks, write_offsets] = vc
        kv.k_scale[write_blocks, write_offsets] = ks
        kv.v_scale[write_blocks, write_offsets] = vs
