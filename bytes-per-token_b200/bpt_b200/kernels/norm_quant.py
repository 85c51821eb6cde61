"""Kernel 1: RMSNorm fused with per-token INT8 activation quantization (`csrc/norm_quant.cu`).

Drop-in for `fastserve.kernels.norm_quant.rms_norm_int8` (`kernels/norm_quant.py:72-109`): the same arguments,
the same result (codes int8 [..., d], scale float32 [..., 1]) and the same `out=(codes [rows, d], scale [rows])`
buffers for allocation-free, graph-captured calls. What it computes is `kernels/reference.py:44-55`:

    y = x / sqrt(mean(x²) + eps) · weight      scale = max(max|y| / 127, 1e-12)      codes = rint(y / scale)

Each row is read once into registers and the three passes run there: from 512 rows of up to 8,192 16-bit values, a
warp per row (eight rows per CTA, persistent CTAs); otherwise a CTA per row. Differences from the reference's
wrapper, none visible in results:
- a view whose rows have unit inner stride (e.g. `x[:, :64]`) is read in place through its row stride; the
  reference copies any non-contiguous input first;
- `num_warps` is accepted for the signature and not used: the launch shape follows rows and d;
- `delta=` adds the decoder layer's residual first (`engine/model.py:109-111`, vLLM's fused add + RMSNorm):
  x + delta, rounded to x's dtype, is normalized, and the sum goes to `x_out` when given.
"""

from __future__ import annotations

import torch

from bpt_b200._lib import FLAG_PDL, check, dtype_code, lib, ptr, require_cuda, stream_of

_FLOATS = (torch.float32, torch.float16, torch.bfloat16)


def rms_norm_int8(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    *,
    out: tuple[torch.Tensor, torch.Tensor] | None = None,
    num_warps: int = 4,
    delta: torch.Tensor | None = None,
    x_out: torch.Tensor | None = None,
    pdl: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm + per-token INT8 in one kernel: (codes int8 [..., d], scale float32 [..., 1]).

    x: [..., d] float32 / float16 / bfloat16 on a CUDA device; weight [d] in any of those dtypes. `out` reuses
    (codes [rows, d], scale [rows]) buffers from an earlier call. With `delta` (x's shape and dtype), x + delta is
    normalized instead and written to `x_out` (contiguous, x's shape and dtype) if that is given.
    """
    del num_warps  # the reference's Triton launch parameter; the block size here follows d
    device = require_cuda(x, weight, delta, x_out, *(out or ()))
    if x.dtype not in _FLOATS:
        raise ValueError(f"rms_norm_int8: x must be float32, float16 or bfloat16, got {x.dtype}")
    d = x.shape[-1]
    rows = x.reshape(-1, d)
    if (d > 1 and rows.stride(-1) != 1) or (rows.shape[0] > 1 and rows.stride(0) < d):
        rows = rows.contiguous()  # rows are read through their stride, elements must be adjacent
    n = rows.shape[0]
    w = weight if weight.dtype in _FLOATS else weight.float()
    if w.numel() != d:
        raise ValueError(f"rms_norm_int8: weight has {w.numel()} elements, rows have {d}")
    w = w.reshape(d).contiguous()
    dflat = None
    if delta is not None:
        if delta.shape != x.shape or delta.dtype != x.dtype:
            raise ValueError("rms_norm_int8: delta must match x in shape and dtype")
        dflat = delta.reshape(n, d).contiguous()
    if x_out is not None:
        if delta is None:
            raise ValueError("rms_norm_int8: x_out holds x + delta and needs delta")
        if x_out.shape != x.shape or x_out.dtype != x.dtype or not x_out.is_contiguous():
            raise ValueError("rms_norm_int8: x_out must be contiguous with x's shape and dtype")
    if out is None:
        out = (
            torch.empty((n, d), dtype=torch.int8, device=device),
            torch.empty(n, dtype=torch.float32, device=device),
        )
    codes, scale = out
    if codes.dtype != torch.int8 or codes.numel() != n * d or not codes.is_contiguous():
        raise ValueError(f"rms_norm_int8: out[0] must be a contiguous int8 buffer of {n} x {d}")
    if scale.dtype != torch.float32 or scale.numel() != n or not scale.is_contiguous():
        raise ValueError(f"rms_norm_int8: out[1] must be a contiguous float32 buffer of {n}")
    st = lib().bpt_rms_norm_int8(
        ptr(rows), dtype_code(x.dtype), rows.stride(0) if n > 1 else d, ptr(w), dtype_code(w.dtype), ptr(dflat),
        ptr(x_out), ptr(codes), ptr(scale), n, d, float(eps), FLAG_PDL if pdl else 0, stream_of(device))
    check(st, "rms_norm_int8")
    return codes.view(x.shape), scale.view(*x.shape[:-1], 1)
