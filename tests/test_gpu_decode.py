"""The Qwen3 decode step (config 5's caller of the hot path) against the oracle, layer by layer.

Each decoder layer is recomputed from the same input hidden state by the reference's arithmetic
(engine/model.py) with the oracle's dequantized W4A16 weights and its paged attention over the same pool; the
KV codes the step writes must equal the oracle's FP8 store bit for bit.
"""

import math

import pytest
import torch

from oracle import attention as oatt
from oracle import kv_formats as okv
from oracle import w4a16 as ow4

pytestmark = pytest.mark.gpu


TOL = {"atol": 1e-2, "rtol": 1e-2}  # the north star's bf16 tolerance


def dequant(t, dense_bf16=False):
    """The layer's dense weight: s (q - z) in fp32, or rounded once to bf16 as the reference model holds it after
    quant/compressed.py:56-69 (what the tcgen05 GEMM multiplies with at M >= 16)."""
    qweight, scales, qzeros = [x.cpu() for x in t]
    n, k = qweight.shape[0], qweight.shape[1] * 8
    g = k // scales.shape[1]
    codes = ow4.unpack_nibbles_int32(qweight, k)
    zeros = ow4.unpack_nibbles_int32(qzeros, k // g)
    w = ow4.dequantize_w4a16(codes, scales, zeros, g)
    return w.to(torch.bfloat16).float() if dense_bf16 else w


def linear(x, w):  # the reference's fp32 linear over the dequantized weight, rounded once to bf16
    return (x.float() @ w.T).to(torch.bfloat16)


def reference_layer(dec, layer, h, cos, sin, lengths_after, kpool, vpool, dense_bf16=False):
    """engine/model.py's DecoderLayer.forward for one token, on the CPU, over the given pools."""
    from bpt_b200.decode import rms_norm, rope_apply

    d = dec.dims
    b = h.shape[0]
    qd, kd = d.q_heads * d.head_dim, d.kv_heads * d.head_dim

    def weight(t):
        return dequant(t, dense_bf16)

    x = rms_norm(h, layer.input_norm.cpu(), d.eps)
    qkv = linear(x, weight(layer.qkv))
    q = rms_norm(qkv[:, :qd].view(b, d.q_heads, d.head_dim), layer.q_norm.cpu(), d.eps)
    k = rms_norm(qkv[:, qd : qd + kd].view(b, d.kv_heads, d.head_dim), layer.k_norm.cpu(), d.eps)
    v = qkv[:, qd + kd :].view(b, d.kv_heads, d.head_dim)
    q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
    kv = okv.PagedKV("fp8", kpool, vpool, layer.kv.k_scale, layer.kv.v_scale, dec.block_table.cpu(), 16)
    attn = oatt.paged_attend(q.float(), kv, lengths_after, 1.0 / math.sqrt(d.head_dim)).to(torch.bfloat16)
    h = h + linear(attn.reshape(b, qd), weight(layer.o))
    x = rms_norm(h, layer.post_norm.cpu(), d.eps)
    gu = weight(layer.gate_up)
    g, u = (x.float() @ gu[0::2].T), (x.float() @ gu[1::2].T)
    act = (torch.nn.functional.silu(g) * u).to(torch.bfloat16)
    return h + linear(act, weight(layer.down)), k, v


def test_decode_step_layers_match_reference():
    from bpt_b200.decode import Qwen3Decoder, Qwen3Dims, rope_cos_sin

    dims = Qwen3Dims(layers=2, intermediate=1024, vocab=512)
    lengths = torch.tensor([40, 17, 100, 64])
    dec = Qwen3Decoder(dims, lengths, seed=3, capacity=8)
    dec.tokens.copy_(torch.tensor([1, 7, 300, 42]))
    b = dec.batch
    pos = dec.lengths.to(torch.int64)
    cos, sin = rope_cos_sin(pos, dims.head_dim, dims.rope_theta, torch.bfloat16)
    write_blocks = torch.gather(dec.block_table, 1, (pos // 16)[:, None]).to(torch.int32)
    write_offsets = (pos % 16).to(torch.int32)[:, None]
    lengths_after = dec.lengths + 1
    h = dec.embed[dec.tokens]
    for layer in dec.layers:
        before_k, before_v = layer.kv.k_pool.cpu(), layer.kv.v_pool.cpu()
        got = dec.layer_forward(layer, h, cos, sin, write_blocks, write_offsets, lengths_after)
        torch.cuda.synchronize()
        kpool, vpool = layer.kv.k_pool.cpu(), layer.kv.v_pool.cpu()
        want, k, v = reference_layer(dec, layer, h.cpu(), cos.cpu(), sin.cpu(), lengths_after.cpu(), kpool, vpool)
        # the step wrote this token's K and V codes, and nothing else. The codes come from the GPU's own k and v,
        # whose last bits can differ from the oracle's (the linear's rounding): a code may sit one E4M3 step from the
        # oracle's store (the write itself is bit-exact from identical inputs: test_gpu_attention.py)
        wb, wo = write_blocks.cpu()[:, 0], write_offsets.cpu()[:, 0]
        for i in range(b):
            for pool, ref, sc in ((kpool, k, layer.kv.k_scale), (vpool, v, layer.kv.v_scale)):
                got_c, want_c = pool[wb[i], wo[i]], okv.fp8_store(ref[i].float(), float(sc))
                assert (got_c == want_c).float().mean() > 0.97
                step = okv.fp8_load(want_c, float(sc)).abs() / 8 + 2 ** -9 * float(sc)  # one E4M3 step, subnormals too
                assert ((okv.fp8_load(got_c, float(sc)) - okv.fp8_load(want_c, float(sc))).abs() <= step * 1.01).all()
            before_k[wb[i], wo[i]] = kpool[wb[i], wo[i]]
            before_v[wb[i], wo[i]] = vpool[wb[i], wo[i]]
        assert torch.equal(before_k, kpool) and torch.equal(before_v, vpool)
        torch.testing.assert_close(got.cpu().float(), want.float(), **TOL)
        h = got


def test_fused_decode_step_batch64_matches_reference():
    """Config 5's benchmarked path: batch 64, so every linear runs on the tcgen05 GEMM, with the fused norm / RoPE
    / KV-write kernels, at Qwen3-1.7B's widths. The residual stream after one decoder layer of an eager step against
    the reference's layer on the CPU (dense bf16 weights, as the tcgen05 GEMM multiplies), atol / rtol 1e-2.

    One layer, compared from the same input: the synthetic pools hold uniformly random E4M3 codes (keys up to
    +-7), so the softmax is sharply peaked and a one-ulp difference in a later layer's input moves its attention
    far more than any kernel error; chaining layers would compare that amplification, not the kernels. (The
    residual stream, not the final-normed output, for the same reason: the final RMSNorm rescales the rounding of
    nearly cancelling elements.)"""
    from bpt_b200.decode import Qwen3Decoder, Qwen3Dims, rope_cos_sin
    from bpt_b200.kernels.w4a16 import w4a16_kernel

    dims = Qwen3Dims(layers=1, vocab=512)
    g = torch.Generator().manual_seed(64)
    lengths = torch.randint(16, 300, (64,), generator=g)
    dec = Qwen3Decoder(dims, lengths, seed=4, capacity=4, fused=True)
    qkv_rows = (dims.q_heads + 2 * dims.kv_heads) * dims.head_dim
    for n, k in ((qkv_rows, dims.hidden), (dims.hidden, dims.q_heads * dims.head_dim),
                 (2 * dims.intermediate, dims.hidden), (dims.hidden, dims.intermediate)):
        assert w4a16_kernel(64, n, k, dims.group) == "tcgen05"
    dec.tokens.copy_(torch.randint(0, dims.vocab, (64,), generator=g))
    pos = dec.lengths.to(torch.int64)
    cos, sin = rope_cos_sin(pos, dims.head_dim, dims.rope_theta, torch.bfloat16)  # as step_body computes them
    lengths_after = (dec.lengths + 1).cpu()
    h = dec.embed[dec.tokens].cpu()
    dec.step()  # eager: embed, the fused layer, final norm, LM head
    torch.cuda.synchronize()
    layer = dec.layers[0]  # its pool now holds the token this step wrote
    want, _, _ = reference_layer(dec, layer, h, cos.cpu(), sin.cpu(), lengths_after, layer.kv.k_pool.cpu(),
                                 layer.kv.v_pool.cpu(), dense_bf16=True)
    torch.testing.assert_close(dec.h.cpu().float(), want.float(), **TOL)  # the fused path's residual stream


def test_decode_step_graph_replay_equals_eager():
    from bpt_b200.decode import Qwen3Decoder, Qwen3Dims

    dims = Qwen3Dims(layers=2, intermediate=1024, vocab=512)
    lengths = torch.tensor([33, 16, 150, 1])
    eager = Qwen3Decoder(dims, lengths, seed=5, capacity=8)
    graphed = Qwen3Decoder(dims, lengths, seed=5, capacity=8)
    graphed.capture()  # one eager step inside, then the capture
    eager.step()
    for _ in range(3):
        eager.step()
        graphed.step()
    torch.cuda.synchronize()
    assert torch.equal(eager.lengths, graphed.lengths)
    assert torch.equal(eager.tokens, graphed.tokens)
    torch.testing.assert_close(eager.hidden.float(), graphed.hidden.float(), atol=0, rtol=0)


def test_fused_rms_norm_residual_matches_reference_ops():
    from bpt_b200.decode import rms_norm
    from bpt_b200.kernels.decode_fused import rms_norm_residual

    g = torch.Generator().manual_seed(7)
    h = (torch.randn(64, 2048, generator=g) * 3).to(torch.bfloat16)
    delta = torch.randn(64, 2048, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16)
    h_out = torch.empty(64, 2048, dtype=torch.bfloat16, device="cuda")
    _, x = rms_norm_residual(h.cuda(), w.cuda(), 1e-6, delta=delta.cuda(), h_out=h_out)
    want_h = h + delta  # the reference's bf16 residual tensor
    assert torch.equal(h_out.cpu(), want_h)
    want = rms_norm(want_h, w, 1e-6)  # engine/model.py:32-35 on the CPU
    got = x.cpu()
    # the fp32 statistics are summed in another order: at most one bf16 step apart, almost always equal
    assert (got.float() - want.float()).abs().max() <= 2 ** -7 * want.float().abs().max()
    assert (got == want).float().mean() > 0.98
    _, x2 = rms_norm_residual(h.cuda(), w.cuda(), 1e-6)  # no residual
    assert (x2.cpu().float() - rms_norm(h, w, 1e-6).float()).abs().max() <= 2 ** -7 * 8


def test_fused_qk_norm_rope_kv_write_matches_reference_ops():
    from bpt_b200.decode import random_e4m3_codes, rms_norm, rope_apply, rope_cos_sin
    from bpt_b200.kernels.decode_fused import qk_norm_rope_kv_write
    from bpt_b200.kernels.kv_attention import PagedQuantKV

    b, hq, hkv, d = 12, 16, 8, 128
    g = torch.Generator().manual_seed(11)
    qkv = torch.randn(b, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    pos = torch.randint(0, 5000, (b,), generator=g)
    cos, sin = rope_cos_sin(pos, d, 1e6, torch.bfloat16)
    pages = 4 * b
    gd = torch.Generator(device="cuda").manual_seed(3)
    kpool = random_e4m3_codes((pages, 16, hkv, d), gd, "cuda")
    vpool = random_e4m3_codes((pages, 16, hkv, d), gd, "cuda")
    table = torch.randperm(pages, generator=g).to(torch.int32).view(b, 4)
    kv = PagedQuantKV("fp8", kpool, vpool, table.cuda(), 16, 1.0 / 64, 1.0 / 32)
    wb = table[:, 1].contiguous()
    wo = torch.randint(0, 16, (b,), generator=g).to(torch.int32)
    before_k, before_v = kpool.cpu(), vpool.cpu()
    q_out = torch.empty(b, hq, d, dtype=torch.bfloat16, device="cuda")
    qk_norm_rope_kv_write(qkv.cuda(), hq, hkv, qn.cuda(), kn.cuda(), cos.cuda(), sin.cuda(), 1e-6, kv, wb.cuda(),
                          wo.cuda(), q_out=q_out)
    # the reference on the CPU: engine/model.py:63-70 with rope.apply, then the FP8 store of the paged write
    q = rope_apply(rms_norm(qkv[:, : hq * d].view(b, hq, d), qn, 1e-6), cos, sin)
    k = rope_apply(rms_norm(qkv[:, hq * d : (hq + hkv) * d].view(b, hkv, d), kn, 1e-6), cos, sin)
    v = qkv[:, (hq + hkv) * d :].view(b, hkv, d)
    got_q = q_out.cpu()
    assert (got_q.float() - q.float()).abs().max() <= 2 ** -6 * q.float().abs().max()
    assert (got_q == q).float().mean() > 0.97
    kp, vp = kpool.cpu(), vpool.cpu()
    for i in range(b):
        # v: no float op in front of the store, so its codes are the oracle's bit for bit
        assert torch.equal(vp[wb[i], wo[i]], okv.fp8_store(v[i].float(), 1.0 / 32))
        want_k = okv.fp8_store(k[i].float(), 1.0 / 64)
        got_k = kp[wb[i], wo[i]]
        assert (got_k == want_k).float().mean() > 0.97  # a norm summed in another order can move a code by one
        assert (okv.fp8_load(got_k, 1.0 / 64) - okv.fp8_load(want_k, 1.0 / 64)).abs().max() <= 2 ** -3 * k[i].float().abs().max()
        before_k[wb[i], wo[i]] = got_k
        before_v[wb[i], wo[i]] = vp[wb[i], wo[i]]
    assert torch.equal(before_k, kp) and torch.equal(before_v, vp)  # nothing else written


def test_fused_decode_step_matches_unfused():
    from bpt_b200.decode import Qwen3Decoder, Qwen3Dims

    dims = Qwen3Dims(layers=3, intermediate=1024, vocab=512)
    lengths = torch.tensor([33, 16, 150, 1, 77, 64])
    plain = Qwen3Decoder(dims, lengths, seed=9, capacity=8, fused=False)
    fused = Qwen3Decoder(dims, lengths, seed=9, capacity=8, fused=True)
    for _ in range(2):
        plain.tokens.copy_(torch.tensor([5, 6, 7, 8, 9, 10]))
        fused.tokens.copy_(plain.tokens)
        plain.step()
        fused.step()
    torch.cuda.synchronize()
    torch.testing.assert_close(fused.hidden.float(), plain.hidden.float(), **TOL)
    assert torch.equal(plain.lengths, fused.lengths)
