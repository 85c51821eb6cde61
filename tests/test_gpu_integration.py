"""The drop-in seams, exercised the way the reference's engine calls them.

- W4A16: `install_w4a16` swaps every decoder linear of a Hugging Face Qwen3 (the module walk and setattr of
  `src/fastserve/quant/model.py:41-47,254-274`), after which the model's own forward runs `W4A16Linear.forward` and
  the fused gate_up MLP. Its logits are compared with the same model on the CPU whose linears hold the oracle's
  dequantized weights (the reference's dequantize-then-nn.Linear path).
- Paged cache: `PagedQuantizedKVCache` is driven through nanoserve's attention seam (`engine/model.py:52-74`:
  prepare once per forward, then `cache.attend(layer, q, k, v, meta, scale)` per layer) for prefill chunks and
  continuous-batching decode steps, against the same seam over the oracle's paged pool on the CPU (the store of
  `kv/quant.py:40-48`, gather-dequantize-attend of `engine/kv_cache.py:165-169` + `kernels/reference.py:186-202`).

The tiny model follows the reference's test fixture (`tests/conftest.py:92-126`: a random transformers Qwen3 with
GQA) at widths these kernels take (hidden 256, head_dim 128, group 128).
"""

import copy
import math

import pytest
import torch

from oracle import attention as oatt
from oracle import kv_formats as okv
from oracle import w4a16 as ow4

pytestmark = pytest.mark.gpu

TOL = {"atol": 1e-2, "rtol": 1e-2}
TINY = {"vocab_size": 512, "hidden_size": 256, "intermediate_size": 512, "num_hidden_layers": 2,
        "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 128, "max_position_embeddings": 512}
LINEARS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def tiny_qwen3(seed=0):
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(seed)
    cfg = transformers.Qwen3Config(**TINY, tie_word_embeddings=False)
    return transformers.Qwen3ForCausalLM._from_config(cfg, attn_implementation="eager").eval()


def sublayer(layer, name):
    return getattr(layer.self_attn if name in LINEARS[:4] else layer.mlp, name)


def oracle_model(model, m_tokens):
    """A CPU fp32 copy of `model` whose decoder linears hold the oracle's dequantized INT4 weights: round_bf16(s (q -
    z)) where the GPU takes the tcgen05 GEMM for M = m_tokens (the reference model's dequantize_linear weight), s (q -
    z) in fp32 where it takes a GEMV (fp32 group sums)."""
    from bpt_b200.kernels.w4a16 import w4a16_kernel

    ref = copy.deepcopy(model).float().cpu()
    for layer in ref.model.layers:
        for name in LINEARS:
            lin = sublayer(layer, name)
            n, k = lin.weight.shape
            codes, scales, zeros = ow4.quantize_w4a16(lin.weight.data.bfloat16().float(), 128)
            w = ow4.dequantize_w4a16(codes, scales, zeros, 128)
            if w4a16_kernel(m_tokens, n, k, 128) == "tcgen05":
                w = w.to(torch.bfloat16).float()
            lin.weight.data.copy_(w)
    return ref


@pytest.mark.parametrize("fuse_gate_up", [True, False])
@pytest.mark.parametrize("batch,seq", [(2, 8), (1, 4)])  # 16 tokens: tcgen05 GEMM; 4 tokens: streaming GEMV
def test_install_w4a16_on_a_hugging_face_qwen3(fuse_gate_up, batch, seq):
    from bpt_b200.kernels.w4a16 import W4A16GateUpMLP, W4A16Linear, install_w4a16

    model = tiny_qwen3().to(torch.bfloat16)
    ref = oracle_model(model, batch * seq)
    model = install_w4a16(model.cuda(), group=128, fuse_gate_up=fuse_gate_up)
    for layer in model.model.layers:
        assert all(isinstance(getattr(layer.self_attn, n), W4A16Linear) for n in LINEARS[:4])
        assert isinstance(layer.mlp, W4A16GateUpMLP) == fuse_gate_up
    ids = torch.randint(0, TINY["vocab_size"], (batch, seq), generator=torch.Generator().manual_seed(seq))
    with torch.no_grad():
        got = model(ids.cuda()).logits.float().cpu()
        want = ref(ids).logits
    torch.testing.assert_close(got, want, **TOL)


# ---- nanoserve's attention seam ------------------------------------------------------------------------------------


def rope(positions, head_dim, theta, dtype):
    """cos, sin [B, Q, D] (engine/rope.py:12-28) for absolute positions [B, Q]."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=positions.device) / head_dim))
    freqs = positions[..., None].float() * inv
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rope_apply(x, cos, sin):  # x [B, H, Q, D]; engine/rope.py:31-43
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos[:, None] + rot * sin[:, None]


def nanoserve_forward(model, ids, positions, cache, rows):
    """engine/model.py:148-170 (CausalLM.forward) with Attention.forward's cache branch (:52-74): the cache's
    prepare once, then cache.attend per layer. `model` is a transformers Qwen3 (same parameter names)."""
    cfg = model.config
    b, q_len = ids.shape
    hd, hq, hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    x = model.model.embed_tokens(ids)
    cos, sin = rope(positions, hd, cfg.rope_parameters["rope_theta"], x.dtype)
    meta = cache.prepare(rows, positions)
    for i, layer in enumerate(model.model.layers):
        at = layer.self_attn
        h = layer.input_layernorm(x)
        q = at.q_norm(at.q_proj(h).view(b, q_len, hq, hd)).transpose(1, 2)
        k = at.k_norm(at.k_proj(h).view(b, q_len, hkv, hd)).transpose(1, 2)
        v = at.v_proj(h).view(b, q_len, hkv, hd).transpose(1, 2)
        q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
        out = cache.attend(i, q, k, v, meta, scale=hd ** -0.5)
        x = x + at.o_proj(out.transpose(1, 2).reshape(b, q_len, -1))
        x = x + layer.mlp(layer.post_attention_layernorm(x))
    return model.lm_head(model.model.norm(x))


class OracleSeamCache:
    """The same seam on the CPU over the oracle's pool (the checker): store with oracle.paged_write, decode with
    gather-dequantize-attend, prefill with a causal attention over the dequantized pages. Shares the GPU cache's
    block tables, so both write the same (block, slot)s.

    follow_gpu: after the store, take the codes (and INT8 scales) the GPU cache wrote into the same slots. A model
    run in bf16 on the GPU and in fp32 here produces k and v that differ in their last bits, and FP8's 3-bit mantissa
    turns such differences into whole code steps (12.5%); comparing the models then needs both sides to attend
    over the same stored codes. (The store itself is checked bit for bit, from identical inputs, by
    test_paged_cache_attend_matches_the_oracle_seam.)"""

    def __init__(self, gpu_cache, follow_gpu=False):
        self.gpu, self.follow_gpu = gpu_cache, follow_gpu
        self.pools = []
        for kv in gpu_cache.layers:
            ks = kv.k_scale if kv.kind == "fp8" else kv.k_scale.cpu().clone()
            vs = kv.v_scale if kv.kind == "fp8" else kv.v_scale.cpu().clone()
            self.pools.append(okv.PagedKV(kv.kind, kv.k_pool.cpu().clone(), kv.v_pool.cpu().clone(), ks, vs,
                                          torch.zeros(0, 1, dtype=torch.int32), kv.block_size))

    def prepare(self, rows, positions):
        meta = self.gpu.prepare(rows, positions.cuda())
        return {k: (getattr(meta, k).cpu() if isinstance(getattr(meta, k), torch.Tensor) else getattr(meta, k))
                for k in ("positions", "write_blocks", "write_offsets", "block_table", "lengths", "kv_len", "q_len")}

    def attend(self, layer, q, k, v, meta, scale):
        kv = self.pools[layer]
        kv.block_table = meta["block_table"]
        wb, wo = meta["write_blocks"].long(), meta["write_offsets"].long()
        okv.paged_write(kv, k.float(), v.float(), wb, wo)
        if self.follow_gpu:
            g = self.gpu.layers[layer]
            kv.k_pool[wb, wo] = g.k_pool.cpu()[wb, wo]
            kv.v_pool[wb, wo] = g.v_pool.cpu()[wb, wo]
            if kv.kind == "int8":
                kv.k_scale[wb, wo] = g.k_scale.cpu()[wb, wo]
                kv.v_scale[wb, wo] = g.v_scale.cpu()[wb, wo]
        if meta["q_len"] == 1:
            return oatt.paged_attend(q[:, :, 0].float(), kv, meta["lengths"], scale)[:, :, None].to(q.dtype)
        kk, vv = oatt.paged_dequantize(kv, meta["kv_len"])
        rep = q.shape[1] // kk.shape[1]
        kk, vv = oatt.repeat_kv(kk, rep), oatt.repeat_kv(vv, rep)
        slots = torch.arange(meta["kv_len"])
        mask = (slots[None, None, :] <= meta["positions"][:, :, None])[:, None]
        s = (q.float() @ kk.transpose(-2, -1)) * scale
        s = s.masked_fill(~mask, float("-inf"))
        return (torch.softmax(s, dim=-1) @ vv).to(q.dtype)


def make_cache(kind, num_layers, decode=None, num_blocks=64):
    from types import SimpleNamespace

    from bpt_b200.integration import PagedQuantizedKVCache

    cfg = SimpleNamespace(num_layers=num_layers, num_kv_heads=2, head_dim=128)
    return PagedQuantizedKVCache(cfg, num_blocks=num_blocks, block_size=16, kind=kind, k_scale=1 / 64, v_scale=1 / 64,
                                 device="cuda", decode=decode)


@pytest.mark.parametrize("kind", ["fp8", "int8"])
@pytest.mark.parametrize("split_decode", [False, True])
def test_paged_cache_attend_matches_the_oracle_seam(kind, split_decode):
    """Random q / k / v through attend: prefill chunks per row (rows at different lengths), then decode steps of
    all rows at their own positions. KV codes bit-exact, fp32 outputs at the reference kernel test's tolerance."""
    from bpt_b200.kernels.kv_attention import decode_attention

    cache = make_cache(kind, 1, decode=decode_attention if split_decode else None)
    ref = OracleSeamCache(cache)
    g = torch.Generator().manual_seed(3)
    lens = {"a": 37, "b": 16, "c": 70}
    for row, n in lens.items():
        cache.reserve(row, n + 8)
    rows = list(lens)

    def step(rows_, positions):
        b, ql = positions.shape
        q = torch.randn(b, 4, ql, 128, generator=g)
        k, v = torch.randn(b, 2, ql, 128, generator=g), torch.randn(b, 2, ql, 128, generator=g)
        meta = cache.prepare(rows_, positions.cuda())
        got = cache.attend(0, q.cuda(), k.cuda(), v.cuda(), meta, scale=1 / math.sqrt(128)).cpu()
        want = ref.attend(0, q, k, v, ref.prepare(rows_, positions), scale=1 / math.sqrt(128))
        torch.testing.assert_close(got, want, rtol=2e-4, atol=2e-4 * want.abs().max().item())
        kv = cache.layers[0]
        assert torch.equal(kv.k_pool.cpu(), ref.pools[0].k_pool) and torch.equal(kv.v_pool.cpu(), ref.pools[0].v_pool)
        if kind == "int8":
            assert torch.equal(kv.k_scale.cpu(), ref.pools[0].k_scale)

    for row, n in lens.items():  # prefill, one row at a time
        step([row], torch.arange(n)[None])
    for i in range(3):  # decode: every row one token further, each at its own position
        step(rows, torch.tensor([[n + i] for n in lens.values()]))


@pytest.mark.parametrize("kind", ["fp8", "int8"])
def test_w4a16_model_with_the_paged_cache_serves_like_the_reference(kind):
    """The whole seam: a Qwen3 with install_w4a16 and a PagedQuantizedKVCache, driven by nanoserve's forward through
    a prefill per prompt and four greedy decode steps of both rows, against the same forward on the CPU over the
    oracle's weights and pool (fed the same tokens). Logits within atol / rtol 1e-2 at every step."""
    from bpt_b200.kernels.w4a16 import install_w4a16

    model = tiny_qwen3(seed=1).to(torch.bfloat16)
    ref_model = oracle_model(model, 6)  # no forward below has more than 6 tokens: all take the GEMV kernels
    model = install_w4a16(model.cuda(), group=128)
    cache = make_cache(kind, TINY["num_hidden_layers"])
    ref_cache = OracleSeamCache(cache, follow_gpu=True)  # the GPU forward of each step runs first
    g = torch.Generator().manual_seed(11)
    prompt = {"r0": 6, "r1": 3}
    for row, n in prompt.items():
        cache.reserve(row, n + 8)
    last = {}
    with torch.no_grad():
        for row, n in prompt.items():  # prefill each prompt (M = n tokens: the GEMV kernels)
            ids = torch.randint(0, TINY["vocab_size"], (1, n), generator=g)
            pos = torch.arange(n)[None]
            got = nanoserve_forward(model, ids.cuda(), pos.cuda(), cache, [row]).float().cpu()
            want = nanoserve_forward(ref_model, ids, pos, ref_cache, [row]).float()
            torch.testing.assert_close(got, want, **TOL)
            last[row] = int(want[0, -1].argmax())
        rows = list(prompt)
        for i in range(4):  # decode all rows together
            ids = torch.tensor([[last[r]] for r in rows])
            pos = torch.tensor([[prompt[r] + i] for r in rows])
            got = nanoserve_forward(model, ids.cuda(), pos.cuda(), cache, rows).float().cpu()
            want = nanoserve_forward(ref_model, ids, pos, ref_cache, rows).float()
            torch.testing.assert_close(got, want, **TOL)
            last = {r: int(want[j, -1].argmax()) for j, r in enumerate(rows)}  # both sides get the same tokens
