"""Oracle: RMSNorm fused with per-token symmetric INT8 quantization, restated on the CPU. TEST INFRASTRUCTURE ONLY.

`rms_norm_int8` follows `src/fastserve/kernels/reference.py:44-55` (the definition the reference's Triton kernel
`kernels/norm_quant.py:42-67` is tested against, `tests/kernels/test_kernels_gpu.py:29-43`):

    y      = x * rsqrt(mean(x^2) + eps) * weight       float32 throughout
    scale  = max(max|y| / 127, 1e-12)                   one per token (row), float32
    codes  = clamp(round(y / scale), -128, 127)         round half to even, int8

With `delta`, the residual add of the model's decoder layer (`src/fastserve/engine/model.py:109-111`) comes
first: h = h + delta in the tensors' own dtype (bf16 in the model), and the sum is what gets normalized.
"""

from __future__ import annotations

import torch

INT8_MAX = 127.0


def rms_norm_int8(x: torch.Tensor, weight: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(codes int8 [..., d], scale float32 [..., 1]); reference.py:44-55, step for step."""
    x32 = x.float()
    y = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    scale = (y.abs().amax(-1, keepdim=True) / INT8_MAX).clamp(min=1e-12)
    codes = torch.clamp(torch.round(y / scale), -128, 127).to(torch.int8)
    return codes, scale


def add_rms_norm_int8(x: torch.Tensor, delta: torch.Tensor, weight: torch.Tensor, eps: float):
    """(h = x + delta in x's dtype, codes, scale): the residual add, then rms_norm_int8 of the sum."""
    h = x + delta
    codes, scale = rms_norm_int8(h, weight, eps)
    return h, codes, scale


def dequantize_int8(codes: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """codes * scale in float32 (reference.py:58-60)."""
    return codes.float() * scale
