"""W4A16: INT4 group-wise weight-only linear layers on sm_100a.

The reference has no W4A16 kernel (production runs vLLM's Marlin; nanoserve dequantizes a checkpoint to dense
BF16 and calls nn.Linear: `src/fastserve/quant/compressed.py:56-69`, `src/fastserve/engine/model.py:43-46`).
This module gives that path a kernel, with the conventions of the reference's kernel module
(`src/fastserve/kernels/norm_quant.py:72-109`): lazy library load, an `out=` buffer for graph capture, and
inputs viewed as [rows, features].

Format (see include/bpt_b200.h):

    qweight  int32 [N, K/8]        code k of row n at bits 4(k mod 8) of word k/8, unsigned 0..15
    scales   fp16  [N, K/group]    qzeros int32 [N, ceil(K/group/8)] (None: symmetric, zero-point 8)

The swap into a model follows the reference's module-swap seam (`src/fastserve/quant/model.py:41-47,254-274`):
`install_w4a16(model)` replaces every decoder linear with a `W4A16Linear` and, optionally, each MLP's
gate/up pair with one fused gate_up + SwiGLU launch.
"""

from __future__ import annotations

import torch
from torch import nn

from bpt_b200 import _lib
from bpt_b200._lib import check, dtype_code, lib, ptr, require_cuda, stream_of

LINEAR_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")  # quant/model.py:32


def quantize_w4a16(w: torch.Tensor, group: int = 128) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """RTN-quantize a dense weight [N, K] (fp32 or bf16, on a CUDA device) on the GPU.

    Asymmetric 4-bit per group of `group` inputs (quant/rtn.py:86-92,113-114) with the scale rounded to fp16
    first (kernels/reference.py:109-114). Returns (qweight int32 [N, K/8], scales fp16 [N, G], qzeros int32
    [N, ceil(G/8)]).
    """
    device = require_cuda(w)
    if w.dim() != 2:
        raise ValueError(f"expected a 2-D weight, got shape {tuple(w.shape)}")
    n, k = w.shape
    if k % group or group % 8:
        raise ValueError(f"{k} input features are not divisible by group size {group}")
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    w = w.contiguous()
    g = k // group
    qweight = torch.empty((n, k // 8), dtype=torch.int32, device=device)
    scales = torch.empty((n, g), dtype=torch.float16, device=device)
    qzeros = torch.empty((n, (g + 7) // 8), dtype=torch.int32, device=device)
    st = lib().bpt_w4a16_quantize(ptr(w), dtype_code(w.dtype), n, k, group, ptr(qweight), ptr(scales), ptr(qzeros),
                                  stream_of(device))
    check(st, "quantize_w4a16")
    return qweight, scales, qzeros


def _rows(x: torch.Tensor, k: int) -> torch.Tensor:
    if x.shape[-1] != k:
        raise ValueError(f"input has {x.shape[-1]} features, the weight expects {k}")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"activations must be bfloat16, got {x.dtype}")
    rows = x.reshape(-1, k)
    if rows.stride(-1) != 1 or rows.stride(0) % 8 or rows.data_ptr() % 16:
        rows = rows.contiguous()
    return rows


def _linear(entry: str, x, qweight, scales, qzeros, group, out, pdl, n_out):
    device = require_cuda(x, qweight, scales, qzeros, out)
    n, k = qweight.shape[0], qweight.shape[1] * 8
    if qweight.dtype != torch.int32 or scales.dtype != torch.float16:
        raise ValueError("qweight must be int32 and scales float16")
    if scales.shape != (n, k // group):
        raise ValueError(f"scales {tuple(scales.shape)} do not match qweight {tuple(qweight.shape)} and group {group}")
    rows = _rows(x, k)
    m = rows.shape[0]
    if out is None:
        out = torch.empty((*x.shape[:-1], n_out), dtype=torch.bfloat16, device=device)
    if out.dtype != torch.bfloat16 or out.shape[-1] != n_out or out.numel() != m * n_out:
        raise ValueError(f"out must be bfloat16 [..., {n_out}] with {m} rows")
    y = out.reshape(m, n_out)
    if m == 0:
        return out
    st = getattr(lib(), entry)(ptr(rows), rows.stride(0), ptr(qweight), ptr(scales), ptr(qzeros), ptr(y), y.stride(0), m,
                               n, k, group, _lib.FLAG_PDL if pdl else 0, stream_of(device))
    check(st, entry)
    return out


def w4a16_linear(x, qweight, scales, qzeros=None, *, group: int = 128, out=None, pdl: bool = False) -> torch.Tensor:
    """y = x . W^T for the packed INT4 weight: x bf16 [..., K] -> bf16 [..., N], fp32 accumulation."""
    return _linear("bpt_w4a16_linear", x, qweight, scales, qzeros, group, out, pdl, qweight.shape[0])


def w4a16_gate_up_silu(x, qweight, scales, qzeros=None, *, group: int = 128, out=None, pdl: bool = False):
    """silu(x . Wg^T) * (x . Wu^T) for a gate/up weight with interleaved rows (see `interleave_rows`)."""
    return _linear("bpt_w4a16_gate_up_silu", x, qweight, scales, qzeros, group, out, pdl, qweight.shape[0] // 2)


KERNELS = {0: "cuda_cores", 1: "mma_gemv", 2: "stream", 3: "mma_gemm", 4: "tcgen05"}


def w4a16_kernel(m: int, n: int, k: int, group: int = 128, zeros: bool = True) -> str:
    """The kernel `w4a16_linear` launches for this shape (16-byte aligned scales and zero points). "tcgen05"
    multiplies with the dense bf16 weight round_bf16(s (q - z)) (the reference's dequantize_linear); the others
    scale each group's fp32 sum of x (q - z)."""
    return KERNELS[int(lib().bpt_w4a16_kernel(m, n, k, group, 1 if zeros else 0))]


def interleave_rows(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[I, ...] and [I, ...] -> [2I, ...] with row 2i = gate row i and row 2i+1 = up row i."""
    if gate.shape != up.shape:
        raise ValueError("gate and up must have the same shape")
    return torch.stack([gate, up], dim=1).reshape(2 * gate.shape[0], *gate.shape[1:])


class W4A16Linear(nn.Module):
    """A bias-free linear layer whose weight is stored as INT4 codes with per-group fp16 scales and zero-points."""

    def __init__(self, qweight, scales, qzeros, group: int = 128):
        super().__init__()
        self.register_buffer("qweight", qweight)
        self.register_buffer("scales", scales)
        self.register_buffer("qzeros", qzeros)
        self.group = group
        self.out_features, self.in_features = qweight.shape[0], qweight.shape[1] * 8

    @classmethod
    def from_linear(cls, linear: nn.Linear, group: int = 128) -> W4A16Linear:
        if linear.bias is not None:
            raise ValueError("W4A16Linear has no bias (Qwen3's linears have none)")
        return cls(*quantize_w4a16(linear.weight.data, group), group=group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return w4a16_linear(x, self.qweight, self.scales, self.qzeros, group=self.group)


class W4A16GateUpMLP(nn.Module):
    """SwiGLU MLP with gate and up fused into one INT4 launch (`engine/model.py:86-96`)."""

    def __init__(self, gate_up: tuple, down: W4A16Linear, group: int = 128):
        super().__init__()
        qweight, scales, qzeros = gate_up
        self.register_buffer("qweight", qweight)
        self.register_buffer("scales", scales)
        self.register_buffer("qzeros", qzeros)
        self.group = group
        self.down_proj = down

    @classmethod
    def from_mlp(cls, mlp: nn.Module, group: int = 128) -> W4A16GateUpMLP:
        gate = quantize_w4a16(mlp.gate_proj.weight.data, group)
        up = quantize_w4a16(mlp.up_proj.weight.data, group)
        fused = tuple(interleave_rows(g, u) for g, u in zip(gate, up, strict=True))
        return cls(fused, W4A16Linear.from_linear(mlp.down_proj, group), group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = w4a16_gate_up_silu(x, self.qweight, self.scales, self.qzeros, group=self.group)
        return self.down_proj(h)


@torch.no_grad()
def install_w4a16(model: nn.Module, group: int = 128, fuse_gate_up: bool = True) -> nn.Module:
    """Swap every decoder linear of a nanoserve / Hugging Face Qwen3 model for its W4A16 version, in place.

    The module walk of quant/model.py:37-47 (`layers[i].self_attn.{q,k,v,o}_proj`, `layers[i].mlp.*`) and the
    setattr swap of quant/model.py:268-274. Embeddings and the LM head stay in 16 bits (quant/model.py:3-4).
    """
    for layer in model.model.layers:
        attn = layer.self_attn
        for name in LINEAR_NAMES[:4]:
            setattr(attn, name, W4A16Linear.from_linear(getattr(attn, name), group))
        if fuse_gate_up:
            layer.mlp = W4A16GateUpMLP.from_mlp(layer.mlp, group)
        else:
            for name in LINEAR_NAMES[4:]:
                setattr(layer.mlp, name, W4A16Linear.from_linear(getattr(layer.mlp, name), group))
    return model
