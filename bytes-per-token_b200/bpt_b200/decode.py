"""A Qwen3 decode step on the hot-path kernels (config 5): the caller of the path, not part of it.

One step takes one new token per sequence through every decoder layer of `engine/model.py` (fastserve's
plain-PyTorch Qwen3): input RMSNorm, the q/k/v projections, QK-norm, RoPE, the KV-cache write, decode
attention over the cache, o_proj and the residual, post-attention RMSNorm, the SwiGLU MLP and its residual;
then the final norm, the tied LM head and a greedy pick. The hot-path pieces run on this package's kernels:

- q, k and v projections as ONE W4A16 linear over the concatenated rows (they share their input), o_proj,
  gate_up fused with SiLU (`w4a16_gate_up_silu`), down_proj;
- the FP8 KV write (`quantize_kv_paged`) at slot `length % 16` of block `block_table[b, length // 16]`;
- paged FP8 decode attention (`attend`, the persistent fused-merge kernel).

With `fused=True` (the default) the small ops around them are two fused kernels per use (`decode_fused.py`):
the residual adds with the following RMSNorm (`engine/model.py:24-36, 109-111`), and q_norm / k_norm, RoPE and
the FP8 cache write of the new token in one pass; `fused=False` runs them as the reference's PyTorch ops (plus
`quantize_kv_paged`). The embedding and the LM head stay in PyTorch. Weights are random (no checkpoints here): N(0, 0.02), quantized to INT4 g128
by `quantize_w4a16`; the LM head stays bf16 and tied to the embedding (`quant/model.py:3-4`). The KV pools hold
random finite E4M3 codes for the existing context. All buffers are allocated up front, so `step` can be
captured in a CUDA graph (`capture`).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from bpt_b200.kernels.decode_fused import qk_norm_rope_kv_write, rms_norm_residual
from bpt_b200.kernels.kv_attention import PagedQuantKV, attend, attend_workspace, paged_split
from bpt_b200.kernels.kv_write import quantize_kv_paged
from bpt_b200.kernels.w4a16 import interleave_rows, quantize_w4a16, w4a16_gate_up_silu, w4a16_linear


@dataclass(frozen=True)
class Qwen3Dims:
    """Qwen3-1.7B (`benchmarks/models/Qwen3-1.7B.config.json`)."""

    hidden: int = 2048
    intermediate: int = 6144
    layers: int = 28
    q_heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1e6
    group: int = 128


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """x / sqrt(mean(x^2) + eps) * weight in float32, cast back before the weight (engine/model.py:32-35)."""
    x32 = x.float()
    x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return weight * x32.to(x.dtype)


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float, dtype: torch.dtype):
    """cos, sin [B, head_dim] for one position per sequence (engine/rope.py:12-28)."""
    exponents = torch.arange(0, head_dim, 2, dtype=torch.float32, device=positions.device) / head_dim
    inv = 1.0 / (theta**exponents)
    freqs = positions[:, None].float() * inv
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, H, D] rotated by rotate-half (engine/rope.py:31-43)."""
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos[:, None] + rot * sin[:, None]


def random_e4m3_codes(shape, generator: torch.Generator, device) -> torch.Tensor:
    """Random E4M3 bytes without the two NaN codes (0x7F, 0xFF), i.e. values a saturating store can produce."""
    codes = torch.randint(0, 256, shape, generator=generator, dtype=torch.uint8, device=device)
    return torch.where((codes & 0x7F) == 0x7F, codes ^ 0x01, codes)


@dataclass
class Layer:
    qkv: tuple  # W4A16 (qweight, scales, qzeros) over [q; k; v] rows
    o: tuple
    gate_up: tuple  # gate and up rows interleaved, for w4a16_gate_up_silu
    down: tuple
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    kv: PagedQuantKV
    dense: dict = field(default_factory=dict)  # the float weights, kept only for checking


class Qwen3Decoder:
    """Random-weight Qwen3 with a paged FP8 cache, stepping `batch` sequences one token at a time.

    `lengths` are the tokens already in each sequence's cache; each step writes one more and attends over
    length + 1. `capacity` is how many steps the block table leaves room for.
    """

    def __init__(self, dims: Qwen3Dims, lengths: torch.Tensor, *, device="cuda", seed: int = 0, capacity: int = 64,
                 kv_scale: float = 1.0 / 64, keep_dense: bool = False, fused: bool = True):
        self.dims, self.device, self.fused = dims, torch.device(device), fused
        d, dev = dims, self.device
        g = torch.Generator(device=dev).manual_seed(seed)
        lengths = lengths.to(torch.int64).cpu()
        self.batch = b = int(lengths.numel())
        self.block_size = 16
        width = int((lengths.max().item() + capacity + 15) // 16)
        pages = int(((lengths + capacity + 15) // 16).sum())
        self.num_blocks = pages
        # each sequence's pages: a random permutation of the pool, shared by all layers (each has its own pool)
        perm = torch.randperm(pages, generator=torch.Generator().manual_seed(seed)).to(torch.int32)
        table = torch.zeros(b, width, dtype=torch.int32)
        pos = 0
        for i, n in enumerate(((lengths + capacity + 15) // 16).tolist()):
            table[i, :n] = perm[pos : pos + n]
            pos += n
        self.block_table = table.to(dev)
        self.lengths = lengths.to(torch.int32).to(dev)  # tokens in the cache before this step
        self.max_tokens = int(lengths.max().item()) + capacity

        def w(n, k):
            return torch.randn(n, k, generator=g, device=dev) * 0.02

        def norm(n):
            return (1.0 + 0.1 * torch.randn(n, generator=g, device=dev)).to(torch.bfloat16)

        self.layers: list[Layer] = []
        qd, kd = d.q_heads * d.head_dim, d.kv_heads * d.head_dim
        for _ in range(d.layers):
            wq, wk, wv = w(qd, d.hidden), w(kd, d.hidden), w(kd, d.hidden)
            wo, wg, wu, wd = w(d.hidden, qd), w(d.intermediate, d.hidden), w(d.intermediate, d.hidden), w(d.hidden, d.intermediate)
            qg, qu = quantize_w4a16(wg, d.group), quantize_w4a16(wu, d.group)
            gate_up = tuple(interleave_rows(x, y) for x, y in zip(qg, qu, strict=True))
            kpool = random_e4m3_codes((pages, 16, d.kv_heads, d.head_dim), g, dev)
            vpool = random_e4m3_codes((pages, 16, d.kv_heads, d.head_dim), g, dev)
            kv = PagedQuantKV("fp8", kpool, vpool, self.block_table, 16, kv_scale, kv_scale)
            layer = Layer(quantize_w4a16(torch.cat([wq, wk, wv]), d.group), quantize_w4a16(wo, d.group), gate_up,
                          quantize_w4a16(wd, d.group), norm(d.hidden), norm(d.hidden), norm(d.head_dim),
                          norm(d.head_dim), kv)
            if keep_dense:
                layer.dense = {"qkv": torch.cat([wq, wk, wv]), "o": wo, "gate": wg, "up": wu, "down": wd}
            self.layers.append(layer)
            del wq, wk, wv, wo, wg, wu, wd
        self.embed = (torch.randn(d.vocab, d.hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        self.final_norm = norm(d.hidden)
        # step buffers (graph-capturable: nothing below allocates outside torch's caching allocator)
        self.tokens = torch.zeros(b, dtype=torch.int64, device=dev)
        self.qkv = torch.empty(b, qd + 2 * kd, dtype=torch.bfloat16, device=dev)
        self.attn = torch.empty(b, d.q_heads, d.head_dim, dtype=torch.bfloat16, device=dev)
        self.proj = torch.empty(b, d.hidden, dtype=torch.bfloat16, device=dev)
        self.act = torch.empty(b, d.intermediate, dtype=torch.bfloat16, device=dev)
        self.h = torch.empty(b, d.hidden, dtype=torch.bfloat16, device=dev)  # residual stream (fused path)
        self.h2 = torch.empty(b, d.hidden, dtype=torch.bfloat16, device=dev)
        self.x = torch.empty(b, d.hidden, dtype=torch.bfloat16, device=dev)  # normed input of the next linear
        self.q = torch.empty(b, d.q_heads, d.head_dim, dtype=torch.bfloat16, device=dev)
        split = paged_split(b, self.max_tokens, 16, torch.cuda.get_device_properties(dev).multi_processor_count)
        self.split = split
        self.workspace = attend_workspace(b, d.q_heads, d.head_dim, -(-self.max_tokens // split), dev).clone()
        self.scale = 1.0 / math.sqrt(d.head_dim)
        self.graph = None

    # ---- one step ----------------------------------------------------------------------------------------------

    def layer_forward(self, layer: Layer, h: torch.Tensor, cos, sin, write_blocks, write_offsets, lengths_after):
        """One decoder layer for one new token per sequence: h [B, hidden] bf16 -> h."""
        d, b = self.dims, self.batch
        qd, kd = d.q_heads * d.head_dim, d.kv_heads * d.head_dim
        x = rms_norm(h, layer.input_norm, d.eps)
        w4a16_linear(x, *layer.qkv, group=d.group, out=self.qkv, pdl=True)
        q = rms_norm(self.qkv[:, :qd].view(b, d.q_heads, d.head_dim), layer.q_norm, d.eps)
        k = rms_norm(self.qkv[:, qd : qd + kd].view(b, d.kv_heads, d.head_dim), layer.k_norm, d.eps)
        v = self.qkv[:, qd + kd :].view(b, d.kv_heads, d.head_dim)
        q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
        quantize_kv_paged(k.unsqueeze(2), v.unsqueeze(2), layer.kv, write_blocks, write_offsets)
        attend(q.contiguous(), layer.kv, lengths_after, self.scale, out=self.attn, workspace=self.workspace,
               tokens=self.max_tokens, split=self.split, pdl=True)
        w4a16_linear(self.attn.view(b, qd), *layer.o, group=d.group, out=self.proj, pdl=True)
        h = h + self.proj
        x = rms_norm(h, layer.post_norm, d.eps)
        w4a16_gate_up_silu(x, *layer.gate_up, group=d.group, out=self.act, pdl=True)
        w4a16_linear(self.act, *layer.down, group=d.group, out=self.proj, pdl=True)
        return h + self.proj

    def layers_fused(self, cos, sin, write_blocks, write_offsets, lengths_after) -> torch.Tensor:
        """Every layer on the fused kernels; self.h holds the embedded tokens. Returns the final-normed hidden.

        Each residual add is fused with the RMSNorm that follows it: the attention residual with the
        post-attention norm, the MLP residual with the next layer's input norm (the final norm after the last)."""
        d, b = self.dims, self.batch
        qd = d.q_heads * d.head_dim
        rms_norm_residual(self.h, self.layers[0].input_norm, d.eps, x_out=self.x, pdl=True)
        for i, layer in enumerate(self.layers):
            w4a16_linear(self.x, *layer.qkv, group=d.group, out=self.qkv, pdl=True)
            qk_norm_rope_kv_write(self.qkv, d.q_heads, d.kv_heads, layer.q_norm, layer.k_norm, cos, sin, d.eps,
                                  layer.kv, write_blocks, write_offsets, q_out=self.q, pdl=True)
            attend(self.q, layer.kv, lengths_after, self.scale, out=self.attn, workspace=self.workspace,
                   tokens=self.max_tokens, split=self.split, pdl=True)
            w4a16_linear(self.attn.view(b, qd), *layer.o, group=d.group, out=self.proj, pdl=True)
            rms_norm_residual(self.h, layer.post_norm, d.eps, delta=self.proj, h_out=self.h2, x_out=self.x, pdl=True)
            w4a16_gate_up_silu(self.x, *layer.gate_up, group=d.group, out=self.act, pdl=True)
            w4a16_linear(self.act, *layer.down, group=d.group, out=self.proj, pdl=True)
            nxt = self.layers[i + 1].input_norm if i + 1 < len(self.layers) else self.final_norm
            rms_norm_residual(self.h2, nxt, d.eps, delta=self.proj, h_out=self.h, x_out=self.x, pdl=True)
        return self.x

    def step_body(self) -> torch.Tensor:
        """Embed self.tokens, run every layer, pick the next tokens (greedy), advance the lengths."""
        d = self.dims
        pos = self.lengths.to(torch.int64)
        cos, sin = rope_cos_sin(pos, d.head_dim, d.rope_theta, torch.bfloat16)
        write_blocks = torch.gather(self.block_table, 1, (pos // self.block_size)[:, None]).to(torch.int32)
        write_offsets = (pos % self.block_size).to(torch.int32)[:, None]
        lengths_after = self.lengths + 1
        if self.fused:
            torch.index_select(self.embed, 0, self.tokens, out=self.h)
            h = self.layers_fused(cos, sin, write_blocks, write_offsets, lengths_after)
        else:
            h = self.embed[self.tokens]
            for layer in self.layers:
                h = self.layer_forward(layer, h, cos, sin, write_blocks, write_offsets, lengths_after)
            h = rms_norm(h, self.final_norm, d.eps)
        logits = h @ self.embed.T
        nxt = logits.argmax(dim=-1)
        self.lengths.add_(1)
        self.tokens.copy_(nxt)
        return h

    def capture(self) -> None:
        """Capture one step in a CUDA graph (after one eager warm-up step, which advances the lengths)."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.step_body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self.hidden = self.step_body()
        torch.cuda.synchronize(self.device)

    def step(self) -> None:
        """One decode step: the captured graph if there is one, else eager."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self.hidden = self.step_body()

    def kv_bytes_per_step(self) -> int:
        """KV bytes one step reads: every layer, every sequence's visible tokens, K and V."""
        d = self.dims
        tokens = int(self.lengths.sum().item()) + self.batch
        return d.layers * tokens * 2 * d.kv_heads * d.head_dim

    def weight_bytes_per_step(self) -> int:
        """INT4 weights (codes + fp16 scales + 4-bit zeros) of every layer, plus the bf16 LM head."""
        d = self.dims
        per_layer = 0
        for n, k in ((d.q_heads * d.head_dim + 2 * d.kv_heads * d.head_dim, d.hidden), (d.hidden, d.q_heads * d.head_dim),
                     (2 * d.intermediate, d.hidden), (d.hidden, d.intermediate)):
            per_layer += n * k // 2 + n * (k // d.group) * 2 + n * (k // d.group) // 2
        return d.layers * per_layer + d.vocab * d.hidden * 2
