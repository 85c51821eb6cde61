"""The CPU oracle against the reference itself: golden vectors made by tests/golden/make_golden.py (which
imports the reference) and the known-answer values of the reference's own tests. CPU only."""

import pytest
import torch

from oracle import attention as oatt
from oracle import kv_formats as okv
from oracle import w4a16 as ow4

# Codes, scales, zero points and packed words are compared bit for bit. Float results of fp32 matmuls and
# softmaxes (y, attention outputs, LSEs) are compared within FLOAT_ORDER: their summation order belongs to the
# host's BLAS kernel, which differs between CPU models, so the golden values (made on one host) move by ulps.
FLOAT_ORDER = {"rtol": 1e-5, "atol": 1e-6}


# ---- W4A16 ------------------------------------------------------------------------------------------------------


def test_rtn_asym_restatement_matches_reference(golden):
    g = golden["rtn_asym"]
    q, scale, zero = ow4.rtn_quantize_asym(g["w"], 4, 128)
    assert torch.equal(q, g["q"]) and torch.equal(scale, g["scale"]) and torch.equal(zero, g["zero"])
    w_hat = ((q - zero) * scale).reshape(g["w"].shape)
    assert torch.equal(w_hat, g["w_hat"])
    torch.testing.assert_close(torch.nn.functional.linear(g["x"], w_hat), g["y"], **FLOAT_ORDER)
    torch.testing.assert_close(g["x"].double() @ w_hat.double().T, g["y"].double(), **FLOAT_ORDER)


def test_stored_grid_is_rtn_with_an_fp16_scale(golden):
    """quantize_w4a16 differs from rtn only by the scale's fp16 rounding: codes within one step, and the
    dequantized weight within half a stored step of the original (plus the fp16 scale's own error)."""
    g = golden["rtn_asym"]
    codes, scales, zeros = ow4.quantize_w4a16(g["w"], 128)
    assert codes.dtype == torch.uint8 and scales.dtype == torch.float16 and zeros.dtype == torch.uint8
    assert int(codes.max()) <= 15 and int(zeros.max()) <= 15
    rtn_q = g["q"].reshape(16, 256)
    assert (codes.int() - rtn_q.int()).abs().max() <= 1
    assert ((codes.int() - rtn_q.int()) != 0).float().mean() < 0.01
    w_hat = ow4.dequantize_w4a16(codes, scales, zeros, 128)
    step = scales.float().repeat_interleave(128, dim=1)
    assert ((w_hat - g["w"]).abs() <= step * (0.51 + 16 * 2**-11)).all()
    assert (w_hat[3, :128] == 0).all()  # an all-zero group dequantizes to exact zeros


def test_unsigned_packing_is_compressed_tensors_pack_int(golden):
    g = golden["pack_int"]
    u = (g["q"].to(torch.int16) + 8).to(torch.uint8)  # pack_int stores q + 8
    assert torch.equal(ow4.pack_nibbles_int32(u), g["packed"])
    assert torch.equal(ow4.pack_nibbles_int32(u[:, :37]), g["packed37"])
    assert torch.equal(ow4.unpack_nibbles_int32(g["packed"], 64).to(torch.int16) - 8, g["unpacked"].to(torch.int16))


def test_symmetric_layout_dequantizes_like_dequantize_linear(golden):
    g = golden["pack_int"]
    codes = ow4.unpack_nibbles_int32(g["packed"], 64)
    dense = ow4.dequantize_w4a16(codes, g["sym_scale"].float(), None, 32)
    assert torch.equal(dense.to(torch.bfloat16), g["dense"])


def test_pack_known_answers():
    """compressed-tensors' layout KATs (reference tests/quant/test_compressed.py:20-26), unsigned form."""
    assert ow4.pack_nibbles_int32(torch.arange(0, 8, dtype=torch.uint8).reshape(1, 8)).item() == 0x76543210
    assert ow4.pack_nibbles_int32(torch.arange(8, 16, dtype=torch.uint8).reshape(1, 8)).item() == 0xFEDCBA98 - 2**32
    every = torch.randint(0, 16, (7, 200), generator=torch.Generator().manual_seed(0), dtype=torch.uint8)
    assert torch.equal(ow4.unpack_nibbles_int32(ow4.pack_nibbles_int32(every), 200), every)


def test_w4a16_linear_from_the_packed_format(golden):
    g = golden["rtn_asym"]
    codes, scales, zeros = ow4.quantize_w4a16(g["w"], 128)
    qweight, scales, qzeros = ow4.pack_w4a16(codes, scales, zeros)
    y = ow4.w4a16_linear(g["x"], qweight, scales, qzeros, 128)
    want = torch.nn.functional.linear(g["x"], ow4.dequantize_w4a16(codes, scales, zeros, 128))
    torch.testing.assert_close(y, want, rtol=0, atol=0)
    torch.testing.assert_close(y, g["y"], rtol=1e-2, atol=1e-2)  # vs rtn's fp32 grid: the fp16 scale only


# ---- KV formats -------------------------------------------------------------------------------------------------


def test_fp8_store_matches_reference_store_and_from_scratch_rounding(golden):
    g = golden["fp8"]
    codes = okv.fp8_store(g["x"], 1.0)
    assert torch.equal(okv.fp8_load(codes, 1.0), g["stored"])
    assert torch.equal(okv.fp8_load(codes, 1.0), g["rounded"])
    assert okv.fp8_load(okv.fp8_store(torch.tensor([1000.0, -1e6]), 1.0), 1.0).tolist() == [448.0, -448.0]


def test_fp8_store_with_a_scale():
    x = torch.randn(1000, generator=torch.Generator().manual_seed(1)) * 3
    codes = okv.fp8_store(x, 0.5)
    assert torch.equal(okv.fp8_load(codes, 0.5), (x / 0.5).to(torch.float8_e4m3fn).float() * 0.5)


def test_fp8_store_keeps_the_sign_of_zero():
    # the reference's cast (kv/quant.py:44-45) maps x / scale of a -0 input to the E4M3 code 0x80, +0 to 0x00; the
    # GPU writes are held to the same codes
    codes = okv.fp8_store(torch.tensor([-0.0, 0.0, -0.0, 1e-30]).to(torch.bfloat16).float(), 0.05)
    assert codes.tolist() == [0x80, 0x00, 0x80, 0x00]


def test_int8_rtn_restatement_matches_reference(golden):
    g = golden["int8_token"]
    q, s = okv.int8_store_rtn(g["x"])
    assert torch.equal(q, g["q"].reshape(64, 128)) and torch.equal(s, g["scale"].reshape(64, 1))
    torch.testing.assert_close(q * s, g["stored"], rtol=0, atol=0)


def test_int8_store_fp16_scale_is_within_one_code_of_rtn(golden):
    g = golden["int8_token"]
    codes, scale = okv.int8_store(g["x"])
    assert codes.dtype == torch.int8 and scale.dtype == torch.float16 and scale.shape == (64,)
    assert (codes.int() - g["q"].reshape(64, 128).int()).abs().max() <= 1
    assert scale[7].item() == 1.0 and (codes[7] == 0).all()  # an all-zero vector: scale 1, codes 0
    err = (okv.int8_load(codes, scale) - g["x"]).abs()
    assert (err <= scale.float()[:, None] * 0.51).all()


@pytest.mark.parametrize("bits", [4, 8, 16])
def test_kivi_restatement_matches_reference(golden, bits):
    g = golden[f"kivi{bits}"]
    kv = okv.kivi_quantize(g["k"], g["v"], bits, 32)
    for name in ("k_codes", "v_codes", "k_scale", "k_zero", "v_scale", "v_zero"):
        if name in g:
            assert torch.equal(getattr(kv, name), g[name]), name
    k_hat, v_hat = okv.kivi_dequantize(kv)
    assert torch.equal(k_hat, g["k_hat"]) and torch.equal(v_hat, g["v_hat"])
    out, lse = oatt.kivi_decode_attention(g["q"], kv, g["lengths"], 0.25)
    torch.testing.assert_close(out, g["out"], **FLOAT_ORDER)
    torch.testing.assert_close(lse, g["lse"], **FLOAT_ORDER)
    torch.testing.assert_close(oatt.merge_partials(out, lse), g["merged"], **FLOAT_ORDER)


def test_nibble_known_answer():
    """reference tests/kernels/test_reference.py:59-65."""
    codes = torch.tensor([[1, 2, 3, 4]], dtype=torch.uint8)
    assert okv.pack_nibbles(codes).tolist() == [[0x31, 0x42]]
    every = torch.arange(16, dtype=torch.uint8).repeat(3, 2)
    assert torch.equal(okv.unpack_nibbles(okv.pack_nibbles(every)), every)


# ---- attention --------------------------------------------------------------------------------------------------


def test_split_merge_matches_reference_with_an_empty_split(golden):
    g = golden["splits"]
    outs, lses = [], []
    for start in (0, 32, 64):
        seen = (g["lengths"] - start).clamp(0, 32)
        o, s = oatt.partial_attention(g["q"], g["k"][:, :, start : start + 32], g["v"][:, :, start : start + 32], seen, 0.25)
        outs.append(o)
        lses.append(s)
    outs, lses = torch.stack(outs, 2), torch.stack(lses, 2)
    torch.testing.assert_close(outs, g["outs"], **FLOAT_ORDER)
    torch.testing.assert_close(lses, g["lses"], **FLOAT_ORDER)
    assert torch.isinf(lses[1, :, 2]).all() and outs[1, :, 2].abs().sum() == 0
    torch.testing.assert_close(oatt.merge_partials(outs, lses), g["merged"], **FLOAT_ORDER)


def test_paged_gather_matches_reference(golden):
    g = golden["paged_gather"]
    got = oatt.paged_gather(g["pool"], g["block_table"], int(g["kv_len"]))
    assert torch.equal(got, g["gathered"])


def test_paged_fp8_attention_matches_reference_pieces(golden):
    g = golden["paged_fp8"]
    kv = okv.PagedKV("fp8", g["k_codes"], g["v_codes"], float(g["k_scale"]), float(g["v_scale"]),
                     g["block_table"], int(g["block_size"]))
    k, v = oatt.paged_dequantize(kv, 17)
    out, lse = oatt.partial_attention(g["q"], k, v, g["lengths"], 0.25)
    torch.testing.assert_close(out, g["out"], **FLOAT_ORDER)
    torch.testing.assert_close(lse, g["lse"], **FLOAT_ORDER)
    # the per-split form merges back to the same answer
    outs, lses = oatt.paged_decode_partials(g["q"], kv, g["lengths"], 0.25, split=8)
    assert outs.shape == (3, 4, 3, 16)
    torch.testing.assert_close(oatt.merge_partials(outs, lses), g["out"], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(oatt.paged_attend(g["q"], kv, g["lengths"], 0.25), g["out"], rtol=1e-6, atol=1e-6)


def test_paged_write_then_gather_round_trips():
    b, hkv, d, bs = 2, 2, 16, 4
    kv = okv.PagedKV("int8", torch.zeros(8, bs, hkv, d, dtype=torch.int8), torch.zeros(8, bs, hkv, d, dtype=torch.int8),
                     torch.zeros(8, bs, hkv, dtype=torch.float16), torch.zeros(8, bs, hkv, dtype=torch.float16),
                     torch.tensor([[5, 2], [7, 0]], dtype=torch.int32), bs)
    k = torch.randn(b, hkv, 6, d, generator=torch.Generator().manual_seed(3))
    pos = torch.arange(6).expand(b, -1)
    blocks = torch.gather(kv.block_table.long(), 1, pos // bs)
    okv.paged_write(kv, k, k * 2, blocks, pos % bs)
    k_hat, v_hat = oatt.paged_dequantize(kv, 6)
    codes, scale = okv.int8_store(k)
    assert torch.equal(k_hat, okv.int8_load(codes, scale))
    assert ((v_hat - 2 * k).abs() <= (2 * k).abs().amax(-1, keepdim=True) / 127 * 0.51 + 1e-6).all()


def test_default_split_golden_values(golden):
    """The reference's default_split (kv_attention.py:178-187), kept by the product's kernel module."""
    from bpt_b200.kernels.kv_attention import default_split

    g = golden["default_split"]
    for case, want in zip(g["cases"].tolist(), g["split"].tolist(), strict=True):
        assert default_split(*case) == want


# ---- RMSNorm + per-token INT8 (kernel 1) ------------------------------------------------------------------------


@pytest.fixture(scope="module")
def norm_golden():
    from conftest import GOLDEN

    return torch.load(GOLDEN.with_name("norm_quant.pt"), weights_only=True)


@pytest.mark.parametrize("name", ["kat", "f32_zero_row", "bf16_3d", "f16_2048", "bf16_x_f32_w", "residual"])
def test_rms_norm_int8_restatement_matches_reference(norm_golden, name):
    """The oracle against reference.rms_norm_int8 (made by tests/golden/make_golden_norm_quant.py): scales within
    FLOAT_ORDER (the row's mean is a host-BLAS sum), codes bit-exact except a code at a rounding tie."""
    from oracle import norm_quant as onq

    g = norm_golden[name]
    if name == "residual":
        h, codes, scale = onq.add_rms_norm_int8(g["h"], g["delta"], g["weight"], float(g["eps"]))
        assert h.dtype == torch.bfloat16 and torch.equal(h, g["x"])
    else:
        codes, scale = onq.rms_norm_int8(g["x"], g["weight"], float(g["eps"]))
    assert codes.dtype == torch.int8 and codes.shape == g["codes"].shape and scale.shape == g["scale"].shape
    torch.testing.assert_close(scale, g["scale"], **FLOAT_ORDER)
    diff = (codes.int() - g["codes"].int()).abs()
    assert diff.max() <= 1 and (diff > 0).float().mean() < 1e-3


def test_rms_norm_int8_known_values(norm_golden):
    """reference tests/kernels/test_reference.py:27-31: y = x / 2.5, scale 1.6 / 127, codes [95, -127, 0, 0]."""
    from oracle import norm_quant as onq

    codes, scale = onq.rms_norm_int8(torch.tensor([[3.0, -4.0, 0.0, 0.0]]), torch.ones(4), 0.0)
    assert codes.tolist() == [[95, -127, 0, 0]] == norm_golden["kat"]["codes"].tolist()
    assert scale.item() == pytest.approx(1.6 / 127)


def test_rms_norm_int8_is_the_model_norm_within_half_a_step(norm_golden):
    """reference tests/kernels/test_reference.py:34-55: codes * scale is the model's RMSNorm within half a step;
    an all-zero token gets zero codes and a finite scale; every other token uses its whole range."""
    from oracle import norm_quant as onq

    g = norm_golden["bf16_3d"]
    codes, scale = onq.rms_norm_int8(g["x"], g["weight"], float(g["eps"]))
    assert ((onq.dequantize_int8(codes, scale) - g["model_norm"]).abs() <= scale / 2 + 1e-5).all()
    z = norm_golden["f32_zero_row"]
    codes, scale = onq.rms_norm_int8(z["x"], z["weight"], float(z["eps"]))
    assert codes[4].abs().sum() == 0 and torch.isfinite(scale).all() and scale[4].item() == pytest.approx(1e-12)
    assert codes.abs().amax(-1)[torch.arange(9) != 4].eq(127).all()
