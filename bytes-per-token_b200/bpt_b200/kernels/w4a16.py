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
gate/up pair with one fused gate_up + SwiGLU launch. `install_w4a16_compressed(model, state, config)` does the
same from a compressed-tensors pack-quantized checkpoint (`from_pack_quantized` per Linear): the checkpoint's
packed words are this format's codes already, so a published INT4 model serves with no dense copy.
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


# ---- compressed-tensors "pack-quantized" checkpoints straight into W4A16 buffers ------------------------------


def from_pack_quantized(tensors: dict[str, torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, None, int]:
    """One Linear of a compressed-tensors pack-quantized (INT4 W4A16) checkpoint -> (qweight, scales, None, group).

    `tensors` holds the module's `weight_packed` int32 [out, in/8], `weight_scale` [out, in/group] and
    `weight_shape` (keys without the module prefix), as `src/fastserve/quant/compressed.py:56-69` reads them. The
    checkpoint's grid is symmetric and each nibble stores q + 8 (`pack_int`, `compressed.py:25-41`): that is this
    module's unsigned code layout with the implicit zero point 8 (`qzeros=None`), so the packed words are used
    as they are and no dense weight is ever built. The scales become fp16; a bf16 scale with magnitude in fp16's
    normal range [2^-14, 65504] converts exactly, and any scale that would change raises ValueError (the
    weights the kernel multiplies are then exactly those `dequantize_linear` builds, before its bf16 rounding).
    """
    if "weight_zero_point" in tensors:
        raise NotImplementedError("asymmetric pack-quantized checkpoints are not read (nor by compressed.py:58-59)")
    if "weight_packed" not in tensors:
        raise ValueError("not a pack-quantized Linear: no weight_packed")
    packed, scale = tensors["weight_packed"], tensors["weight_scale"]
    out, cols = (int(v) for v in tensors["weight_shape"])
    if packed.dtype != torch.int32 or packed.dim() != 2 or packed.shape[0] != out or packed.shape[1] * 8 < cols:
        raise ValueError(f"weight_packed must be int32 [{out}, {(cols + 7) // 8}], got {tuple(packed.shape)}")
    if cols % 8 != 0 or packed.shape[1] * 8 != cols:
        raise ValueError(f"input features {cols} must fill whole int32 words (a multiple of 8)")
    if scale.dim() != 2 or scale.shape[0] != out or cols % scale.shape[1] != 0:
        raise ValueError(f"weight_scale must be [{out}, groups] with groups dividing {cols}")
    group = cols // scale.shape[1]
    scales = scale.to(torch.float16)
    if not torch.equal(scales.to(scale.dtype), scale) or not torch.isfinite(scales).all():
        raise ValueError("weight_scale does not convert exactly to fp16 (a scale outside fp16's normal range)")
    return packed.contiguous(), scales.contiguous(), None, group


def _pack_quantized_parts(state: dict[str, torch.Tensor], module: str) -> dict[str, torch.Tensor]:
    parts = {n: state[f"{module}.{n}"] for n in ("weight_packed", "weight_scale", "weight_shape", "weight_zero_point")
             if f"{module}.{n}" in state}
    if "weight_packed" not in parts:
        raise ValueError(f"{module}: no weight_packed in the checkpoint")
    return parts


@torch.no_grad()
def install_w4a16_compressed(model: nn.Module, state: dict[str, torch.Tensor], quantization_config: dict,
                             fuse_gate_up: bool = True, prefix: str = "model.layers") -> nn.Module:
    """`install_w4a16` fed from a pack-quantized checkpoint's state dict instead of dense weights: every decoder
    linear of the model becomes a W4A16Linear over the checkpoint's own codes and scales (and each gate/up pair
    one fused launch, their rows interleaved), so a published INT4 checkpoint serves without the dense BF16 copy
    that `compressed.dense_state_dict` (`compressed.py:72-97`) builds. Buffers land on each module's device."""
    if quantization_config.get("format") != "pack-quantized":
        raise ValueError(f"expected a pack-quantized checkpoint, got format {quantization_config.get('format')!r}")
    bits = {g["weights"]["num_bits"] for g in quantization_config["config_groups"].values()}
    if bits != {4}:
        raise NotImplementedError(f"4-bit weights expected, got {sorted(bits)}")
    for i, layer in enumerate(model.model.layers):
        def load(sub: str, name: str, like: nn.Module):
            qw, sc, _, group = from_pack_quantized(_pack_quantized_parts(state, f"{prefix}.{i}.{sub}.{name}"))
            device = next(like.parameters()).device
            return qw.to(device), sc.to(device), group

        attn = layer.self_attn
        for name in LINEAR_NAMES[:4]:
            qw, sc, group = load("self_attn", name, getattr(attn, name))
            setattr(attn, name, W4A16Linear(qw, sc, None, group))
        mlp = layer.mlp
        if fuse_gate_up:
            gq, gs, group = load("mlp", "gate_proj", mlp.gate_proj)
            uq, us, group_up = load("mlp", "up_proj", mlp.up_proj)
            if group_up != group:
                raise ValueError("gate_proj and up_proj must share a group size to be fused")
            dq, ds, dgroup = load("mlp", "down_proj", mlp.down_proj)
            layer.mlp = W4A16GateUpMLP((interleave_rows(gq, uq), interleave_rows(gs, us), None),
                                       W4A16Linear(dq, ds, None, dgroup), group)
        else:
            for name in LINEAR_NAMES[4:]:
                qw, sc, group = load("mlp", name, getattr(mlp, name))
                setattr(mlp, name, W4A16Linear(qw, sc, None, group))
    return model
