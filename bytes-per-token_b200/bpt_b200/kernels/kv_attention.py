"""Decode attention over a quantized KV cache, on sm_100a, with the reference kernel module's signatures.

Mirrors `src/fastserve/kernels/kv_attention.py` (ish-codes-magic/bytes-per-token):

    default_split(batch, kv_heads, tokens, group=32, max_programs=16384)      (kv_attention.py:178-187)
    decode_attention(q, kv, lengths, scale, *, tokens=None, split=None, num_warps=1)
        -> (out [B, Hq, S, D] f32, lse [B, Hq, S] f32)                          (kv_attention.py:190-245)
    attend(q, kv, lengths, scale, **launch) -> [B, Hq, D] f32                  (kv_attention.py:248-252)

`kv` is either the reference's contiguous KIVI cache (any object with QuantKV's fields: bits, group, k_codes,
v_codes, k_scale, k_zero, v_scale, v_zero; `QuantKV` below has them) or a `PagedQuantKV`: the paged FP8 / INT8
pool this build adds, in the reference's paged layout [num_blocks, block_size, Hkv, D]
(`src/fastserve/engine/kv_cache.py:108`). The same functions serve both, so the cache that calls them
(`QuantizedKVCache.attend`, `integration/kv_cache.py:160-185`) does not change.

Every path runs a CUDA kernel from libbpt_b200.so; tensors must be on a CUDA device. `num_warps` is accepted
for signature compatibility and ignored (the launch shapes are fixed per kernel). `split % group != 0`
raises ValueError, as in the reference (kv_attention.py:216-217).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from bpt_b200 import _lib
from bpt_b200._lib import check, dtype_code, lib, ptr, require_cuda, stream_of


@dataclass
class QuantKV:
    """The reference's contiguous KIVI cache (kernels/reference.py:66-100), same fields and shapes:

    k_codes, v_codes  [B, Hkv, T, D] (bits 8, 16) or [B, Hkv, T, D/2] (bits 4, channel d low / d + D/2 high)
    k_scale, k_zero   [B, Hkv, T/group, D] fp16       v_scale, v_zero [B, Hkv, T] fp16
    """

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

    @property
    def head_dim(self) -> int:
        return self.k_codes.shape[3] * (2 if self.bits == 4 else 1)


@dataclass
class PagedQuantKV:
    """One layer's paged, quantized KV cache.

    kind         "fp8": E4M3 bytes (uint8), k_scale / v_scale are per-tensor floats
                 "int8": int8 codes, k_scale / v_scale are fp16 [num_blocks, block_size, Hkv] (one per token, head)
    k_pool/v_pool [num_blocks, block_size, Hkv, D]
    block_table  int32 [B, n_blocks]: physical block of each sequence's logical block j (tokens j*bs .. j*bs+bs-1)
    """

    kind: str
    k_pool: torch.Tensor
    v_pool: torch.Tensor
    block_table: torch.Tensor
    block_size: int
    k_scale: float | torch.Tensor = 1.0
    v_scale: float | torch.Tensor = 1.0

    @property
    def tokens(self) -> int:
        """Tokens the block table can address per sequence (its width times the block size)."""
        return self.block_table.shape[1] * self.block_size

    @property
    def head_dim(self) -> int:
        return self.k_pool.shape[3]

    @property
    def kv_heads(self) -> int:
        return self.k_pool.shape[2]

    @property
    def num_blocks(self) -> int:
        return self.k_pool.shape[0]

    def bytes_per_token(self) -> float:
        """Bytes one token occupies across this layer's KV heads, scales included."""
        per = 2 * self.kv_heads * self.head_dim
        return float(per + (2 * self.kv_heads * 2 if self.kind == "int8" else 0))


def default_split(batch: int, kv_heads: int, tokens: int, group: int = 32, max_programs: int = 16384) -> int:
    """Tokens per program for the KIVI kernel: the reference's rule (kv_attention.py:178-187), unchanged."""
    per_program = max(tokens * batch * kv_heads // max_programs, 4 * group)
    return max(group, 1 << (per_program.bit_length() - 1))


def kivi_attend_split(batch: int, kv_heads: int, tokens: int, group: int = 32) -> int:
    """Tokens per program when only the merged result is wanted (`attend` over a KIVI cache): the longest power of
    two up to 512 that still leaves 512 programs, and at least 4 key groups. Longer splits than the reference's
    rule (`default_split`, kept by `decode_attention`, whose per-split outputs depend on it) mean fewer partials to
    write and merge: 8 x 32k INT4 measured 234 -> 194 us at 512 tokens against 128."""
    split = 512
    while split > 4 * group and batch * kv_heads * -(-tokens // split) < 512:
        split //= 2
    return max(split, 4 * group)


def paged_split(batch: int, tokens: int, block_size: int = 16, sms: int = 148) -> int:
    """Tokens per CTA for the paged kernel, whose CTA covers every KV head of one sequence's split.

    About four CTAs per SM at the longest length (fewer with ragged lengths), as a power of two between
    4 pages and 64 pages; enough splits that one long sequence still fills the GPU.
    """
    target = max(batch * tokens // (4 * sms), 1)
    split = 1 << (target.bit_length() - 1)
    return int(min(max(split, 4 * block_size), 64 * block_size))


def _sms(device: torch.device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def _q_view(q: torch.Tensor) -> torch.Tensor:
    return q if q.stride(-1) == 1 else q.contiguous()


def _lengths(lengths: torch.Tensor) -> torch.Tensor:
    return lengths if lengths.dtype == torch.int32 and lengths.is_contiguous() else lengths.to(torch.int32).contiguous()


def _paged_args(q: torch.Tensor, kv: PagedQuantKV):
    if kv.kind not in ("fp8", "int8"):
        raise ValueError(f"kind must be 'fp8' or 'int8', got {kv.kind!r}")
    b, hq, d = q.shape
    nb, bs, hkv, dk = kv.k_pool.shape
    if dk != d or kv.v_pool.shape != kv.k_pool.shape:
        raise ValueError(f"pool shape {tuple(kv.k_pool.shape)} does not match q {tuple(q.shape)}")
    if kv.block_table.shape[0] != b:
        raise ValueError(f"block table has {kv.block_table.shape[0]} rows for a batch of {b}")
    if kv.block_table.dtype != torch.int32:
        raise ValueError("the block table must be int32")
    if kv.kind == "fp8":
        ks, vs, kss, vss = float(kv.k_scale), float(kv.v_scale), None, None
        code = _lib.KV_FP8
    else:
        kss, vss = kv.k_scale, kv.v_scale
        if not (isinstance(kss, torch.Tensor) and kss.dtype == torch.float16 and tuple(kss.shape) == (nb, bs, hkv)):
            raise ValueError("int8 pools need fp16 k_scale / v_scale of shape [num_blocks, block_size, Hkv]")
        ks = vs = 1.0
        code = _lib.KV_INT8
    return code, ks, vs, kss, vss, nb, bs, hkv


def decode_attention(
    q: torch.Tensor,
    kv: QuantKV | PagedQuantKV,
    lengths: torch.Tensor,
    scale: float,
    *,
    tokens: int | None = None,
    split: int | None = None,
    num_warps: int = 1,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Partial attentions of one query per head over a quantized cache, one per split of `split` tokens.

    q [B, Hq, D] (fp32, fp16 or bf16); lengths [B] int32. `tokens` bounds the launch when the caller knows the
    longest length (no host sync on lengths.max()). Returns (out [B, Hq, S, D], lse [B, Hq, S]) in fp32; a split
    past a row's end has out 0 and lse -inf, so `merge_partials` ignores it.
    """
    del num_warps
    device = require_cuda(q, lengths, kv.k_codes if not isinstance(kv, PagedQuantKV) else kv.k_pool)
    q = _q_view(q)
    lengths = _lengths(lengths)
    b, hq, d = q.shape
    if isinstance(kv, PagedQuantKV):
        code, ks, vs, kss, vss, nb, bs, hkv = _paged_args(q, kv)
        tokens = kv.tokens if tokens is None else tokens
        if split is None:
            split = paged_split(b, tokens, bs, _sms(device))
        if split % bs:
            raise ValueError(f"split {split} must be a multiple of the block size {bs}")
        n_splits = max(-(-tokens // split), 1)
        out = torch.empty((b, hq, n_splits, d), dtype=torch.float32, device=device)
        lse = torch.empty((b, hq, n_splits), dtype=torch.float32, device=device)
        st = lib().bpt_paged_decode_partials(
            ptr(q), dtype_code(q.dtype), q.stride(0), q.stride(1), ptr(kv.k_pool), ptr(kv.v_pool), code, ks, vs,
            ptr(kss), ptr(vss), ptr(kv.block_table), kv.block_table.stride(0), ptr(lengths), b, hq, hkv, d, bs, nb,
            split, n_splits, float(scale), ptr(out), ptr(lse), 0, stream_of(device))
        check(st, "decode_attention (paged)")
        return out, lse

    kv_heads, t_max = kv.k_codes.shape[1], kv.k_codes.shape[2]
    tokens = t_max if tokens is None else tokens
    if split is None:
        split = default_split(b, kv_heads, tokens, kv.group)
    if split % kv.group:
        raise ValueError(f"split {split} must be a multiple of the key group {kv.group}")
    n_splits = max(-(-tokens // split), 1)
    out = torch.empty((b, hq, n_splits, d), dtype=torch.float32, device=device)
    lse = torch.empty((b, hq, n_splits), dtype=torch.float32, device=device)
    n_groups = kv.k_scale.shape[2] if kv.k_scale is not None else -(-t_max // kv.group)
    code_dtype = dtype_code(kv.k_codes.dtype) if kv.bits == 16 else 0
    st = lib().bpt_kivi_decode_partials(
        ptr(q), dtype_code(q.dtype), q.stride(0), q.stride(1), kv.bits, code_dtype, ptr(kv.k_codes), ptr(kv.v_codes),
        ptr(kv.k_scale), ptr(kv.k_zero), ptr(kv.v_scale), ptr(kv.v_zero), ptr(lengths), b, hq, kv_heads, d, t_max,
        n_groups, kv.group, split, n_splits, float(scale), ptr(out), ptr(lse), stream_of(device))
    check(st, "decode_attention (KIVI)")
    return out, lse


def merge_partials(outs: torch.Tensor, lses: torch.Tensor, out_dtype: torch.dtype = torch.float32, *,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """[B, Hq, S, D], [B, Hq, S] -> [B, Hq, D]: the exact merge of split partials (reference.py:205-211).

    `out` (contiguous [B, Hq, D], float32 / float16 / bfloat16) receives the result in its own dtype instead of a
    new tensor of `out_dtype`."""
    device = require_cuda(outs, lses, out)
    if outs.dtype != torch.float32 or lses.dtype != torch.float32:
        raise ValueError("partials must be float32")
    outs, lses = outs.contiguous(), lses.contiguous()
    b, hq, s, d = outs.shape
    if out is not None:
        if tuple(out.shape) != (b, hq, d) or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous [{b}, {hq}, {d}] tensor")
        merged, out_dtype = out, out.dtype
    else:
        merged = torch.empty((b, hq, d), dtype=out_dtype, device=device)
    st = lib().bpt_merge_partials(ptr(outs), ptr(lses), b, hq, s, d, ptr(merged), dtype_code(out_dtype), stream_of(device))
    check(st, "merge_partials")
    return merged


_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def attend_workspace(batch: int, q_heads: int, head_dim: int, n_splits: int, device: torch.device) -> torch.Tensor:
    """A zeroed workspace for the fused split merge, cached per device and stream, grown on demand.

    Each call of the fused kernel leaves the workspace's counters at zero again, so the buffer is reused as is.
    Calls that overlap on the GPU (different streams) need different workspaces: the cache is keyed by stream.
    Under CUDA graph capture, size it before capturing (or pass `workspace=` to `attend`).
    """
    need = int(lib().bpt_paged_attend_workspace_bytes(batch, q_heads, head_dim, n_splits))
    key = (device.index or 0, stream_of(device))
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(max(need, 1 << 16), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def attend(
    q: torch.Tensor,
    kv: QuantKV | PagedQuantKV,
    lengths: torch.Tensor,
    scale: float,
    *,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    **launch,
) -> torch.Tensor:
    """Decode attention over a quantized cache: [B, Hq, D] (fp32 unless `out` says otherwise).

    Paged caches run one fused launch: the splits of a sequence are merged by the last of its CTAs to finish.
    KIVI caches run the split kernel, then the merge kernel. `pdl=True` launches with programmatic dependent
    launch; `kv_ready=True` adds the promise that the lengths, block table and pools are not written by the
    kernel this call follows, so the persistent kernel starts copying pages before it waits on that kernel.
    """
    if not isinstance(kv, PagedQuantKV):  # the merge writes straight into `out` when one is given
        if launch.get("split") is None:
            launch = dict(launch, split=kivi_attend_split(q.shape[0], kv.k_codes.shape[1],
                                                           launch.get("tokens") or kv.k_codes.shape[2], kv.group))
        return merge_partials(*decode_attention(q, kv, lengths, scale, **launch), out=out)
    device = require_cuda(q, lengths, kv.k_pool)
    q = _q_view(q)
    lengths = _lengths(lengths)
    b, hq, d = q.shape
    code, ks, vs, kss, vss, nb, bs, hkv = _paged_args(q, kv)
    tokens = launch.get("tokens") or kv.tokens
    split = launch.get("split") or paged_split(b, tokens, bs, _sms(device))
    if split % bs:
        raise ValueError(f"split {split} must be a multiple of the block size {bs}")
    n_splits = max(-(-tokens // split), 1)
    if out is None:
        out = torch.empty((b, hq, d), dtype=torch.float32, device=device)
    if tuple(out.shape) != (b, hq, d) or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous [{b}, {hq}, {d}] tensor")
    if workspace is None:
        workspace = attend_workspace(b, hq, d, n_splits, device)
    st = lib().bpt_paged_attend(
        ptr(q), dtype_code(q.dtype), q.stride(0), q.stride(1), ptr(kv.k_pool), ptr(kv.v_pool), code, ks, vs, ptr(kss),
        ptr(vss), ptr(kv.block_table), kv.block_table.stride(0), ptr(lengths), b, hq, hkv, d, bs, nb, split, n_splits,
        float(scale), ptr(out), dtype_code(out.dtype), ptr(workspace), workspace.numel(),
        (_lib.FLAG_PDL if launch.get("pdl") else 0) | (_lib.FLAG_KV_READY if launch.get("kv_ready") else 0),
        stream_of(device))
    check(st, "attend (paged)")
    return out


def sm_scale(head_dim: int) -> float:
    """The model's softmax scale, head_dim^-0.5 (engine/model.py:73)."""
    return 1.0 / math.sqrt(head_dim)
