"""The contiguous KIVI path (the reference's own cache layout and decode_attention signature) against the CPU
oracle, on the shapes of the reference's GPU tests (tests/kernels/test_kernels_gpu.py:87-142), and the GPU KIVI
quantizer bit for bit against oracle.kv_formats.kivi_quantize."""

import pytest
import torch

from oracle import attention as oatt
from oracle import kv_formats as okv

pytestmark = pytest.mark.gpu


def rand(*shape, seed=0, dtype=torch.float32):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)).to(dtype)


def quantized(batch, kv_heads, tokens, d, bits, seed=0, dtype=torch.bfloat16):
    k = rand(batch, kv_heads, tokens, d, seed=seed, dtype=dtype)
    k[..., 3 % d] += 20.0  # an outlier channel, as Qwen3's keys have
    v = rand(batch, kv_heads, tokens, d, seed=seed + 1, dtype=dtype)
    return k, v, okv.kivi_quantize(k, v, bits)


def to_gpu(kv):
    from bpt_b200.kernels.kv_attention import QuantKV

    f = (lambda t: None if t is None else t.cuda())
    return QuantKV(kv.bits, kv.group, f(kv.k_codes), f(kv.v_codes), f(kv.k_scale), f(kv.k_zero), f(kv.v_scale),
                   f(kv.v_zero))


def check_attention(q, kv_cpu, kv_gpu, lengths, scale=0.1, **launch):
    from bpt_b200.kernels.kv_attention import attend

    got = attend(q.cuda(), kv_gpu, lengths.cuda(), scale, **launch).cpu()
    want = oatt.merge_partials(*oatt.kivi_decode_attention(q, kv_cpu, lengths, scale))
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got, want, rtol=2e-4, atol=2e-4 * want.abs().max().item())


@pytest.mark.parametrize("bits", [4, 8, 16])
@pytest.mark.parametrize(
    "batch,q_heads,kv_heads,tokens,d",
    [(1, 16, 8, 32, 128), (2, 16, 8, 96, 128), (3, 4, 2, 160, 16), (2, 4, 4, 64, 32), (1, 16, 8, 4096, 128)],
)
def test_attention_matches_oracle(batch, q_heads, kv_heads, tokens, d, bits):
    for seed in range(2):
        _, _, kv = quantized(batch, kv_heads, tokens, d, bits, seed=seed)
        kv_gpu = to_gpu(kv)
        q = rand(batch, q_heads, d, seed=seed + 7)
        full = torch.full((batch,), tokens, dtype=torch.int32)
        check_attention(q, kv, kv_gpu, full)
        for split in (32, 64, tokens):
            check_attention(q, kv, kv_gpu, full, split=split)
        check_attention(q, kv, kv_gpu, full, split=32, num_warps=8)


@pytest.mark.parametrize("bits", [4, 8, 16])
def test_attention_respects_each_rows_length(bits):
    from bpt_b200.kernels.kv_attention import attend

    _, _, kv = quantized(4, 8, 160, 128, bits)
    kv_gpu = to_gpu(kv)
    q = rand(4, 16, 128, seed=3)
    lengths = torch.tensor([160, 1, 70, 0], dtype=torch.int32)
    check_attention(q, kv, kv_gpu, lengths, split=64)
    check_attention(q, kv, kv_gpu, lengths, tokens=160)
    assert attend(q.cuda(), kv_gpu, lengths.cuda(), 0.1, split=32)[3].abs().sum() == 0


def test_attention_other_dtypes_and_a_shorter_launch():
    _, _, kv = quantized(2, 8, 128, 128, 16, dtype=torch.float16)
    q = rand(2, 16, 128, seed=4, dtype=torch.float16)
    lengths = torch.tensor([64, 64], dtype=torch.int32)
    check_attention(q, kv, to_gpu(kv), lengths)
    check_attention(q, kv, to_gpu(kv), lengths, tokens=64)


def test_attention_at_max_context():
    _, _, kv = quantized(1, 8, 32768, 128, 4)
    kv_gpu = to_gpu(kv)
    q = rand(1, 16, 128, seed=9)
    check_attention(q, kv, kv_gpu, torch.tensor([32768], dtype=torch.int32))
    check_attention(q, kv, kv_gpu, torch.tensor([32001], dtype=torch.int32), split=2048)


def test_decode_attention_returns_the_reference_contract():
    from bpt_b200.kernels.kv_attention import decode_attention

    _, _, kv = quantized(2, 8, 96, 128, 8)
    q = rand(2, 16, 128, seed=5)
    lengths = torch.tensor([96, 40], dtype=torch.int32)
    out, lse = decode_attention(q.cuda(), to_gpu(kv), lengths.cuda(), 0.1, split=32)
    assert out.shape == (2, 16, 3, 128) and lse.shape == (2, 16, 3) and out.dtype == torch.float32
    assert torch.isinf(lse[1, :, 2]).all() and out[1, :, 2].abs().sum() == 0  # past row 1's end
    with pytest.raises(ValueError, match="multiple of the key group"):
        decode_attention(q.cuda(), to_gpu(kv), lengths.cuda(), 0.1, split=48)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("d", [16, 32, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_kivi_quantize_is_bit_exact(bits, d, dtype):
    from bpt_b200.kernels.kv_write import quantize_kv

    k, v, want = quantized(2, 3, 96, d, bits, seed=d, dtype=dtype)
    got = quantize_kv(k.cuda(), v.cuda(), bits)
    for name in ("k_codes", "v_codes", "k_scale", "k_zero", "v_scale", "v_zero"):
        assert torch.equal(getattr(got, name).cpu(), getattr(want, name)), name


def test_kivi_quantize_into_a_larger_cache_at_an_offset():
    from bpt_b200.kernels.kv_write import empty_quant_kv, quantize_kv_into

    k, v, want = quantized(2, 2, 64, 128, 4, seed=11)
    cache = empty_quant_kv(2, 2, 128, 128, 4, 32, "cuda")
    quantize_kv_into(k.cuda(), v.cuda(), cache, 32)
    assert torch.equal(cache.k_codes[:, :, 32:96].cpu(), want.k_codes)
    assert torch.equal(cache.k_scale[:, :, 1:3].cpu(), want.k_scale)
    assert torch.equal(cache.v_zero[:, :, 32:96].cpu(), want.v_zero)
    assert cache.k_codes[:, :, :32].abs().sum() == 0 and cache.k_codes[:, :, 96:].abs().sum() == 0
