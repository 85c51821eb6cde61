"""rms_norm_int8 (RMSNorm + per-token INT8, `csrc/norm_quant.cu`) against the CPU oracle `oracle/norm_quant.py`
and the reference's golden outputs, with the reference's own GPU-test tolerances
(`tests/kernels/test_kernels_gpu.py:29-66`): scales within rtol 1e-5, codes equal except a value at a rounding tie
whose row sums differ in the last bit (at most one code apart, under 0.1% of the codes)."""

import pytest
import torch

from oracle import norm_quant as onq

pytestmark = pytest.mark.gpu

FLOATS = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def rand(*shape, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


def check(codes, scale, want_codes, want_scale):
    assert codes.dtype == torch.int8 and codes.shape == want_codes.shape and scale.shape == want_scale.shape
    torch.testing.assert_close(scale.cpu(), want_scale, rtol=1e-5, atol=0)
    diff = (codes.cpu().int() - want_codes.int()).abs()
    assert diff.max() <= 1 and (diff > 0).float().mean() < 1e-3


@pytest.mark.parametrize("dtype", list(FLOATS))
@pytest.mark.parametrize("rows,d", [(1, 1024), (3, 2048), (257, 1000), (64, 3), (5, 1), (4096, 1024), (64, 2048)])
def test_rms_norm_int8_matches_oracle(rows, d, dtype):
    from bpt_b200.kernels.norm_quant import rms_norm_int8

    for seed in range(3):
        x = rand(rows, d, seed=seed, dtype=FLOATS[dtype]) * 3
        weight = (rand(d, seed=seed + 100).abs() + 0.5).to(FLOATS[dtype])
        codes, scale = rms_norm_int8(x.cuda(), weight.cuda(), 1e-6)
        assert scale.shape == (rows, 1)
        check(codes, scale, *onq.rms_norm_int8(x, weight, 1e-6))


@pytest.mark.parametrize("name", ["kat", "f32_zero_row", "bf16_3d", "f16_2048", "bf16_x_f32_w"])
def test_rms_norm_int8_matches_reference_goldens(name):
    from conftest import GOLDEN

    from bpt_b200.kernels.norm_quant import rms_norm_int8

    g = torch.load(GOLDEN.with_name("norm_quant.pt"), weights_only=True)[name]
    codes, scale = rms_norm_int8(g["x"].cuda(), g["weight"].cuda(), float(g["eps"]))
    check(codes, scale, g["codes"], g["scale"])
    if name == "kat":  # reference tests/kernels/test_reference.py:27-31, bit for bit
        assert codes.cpu().tolist() == [[95, -127, 0, 0]]
        assert scale.item() == onq.rms_norm_int8(g["x"], g["weight"], 0.0)[1].item()


def test_rms_norm_int8_shapes_views_zero_rows_and_out_buffers():
    """reference tests/kernels/test_kernels_gpu.py:46-66."""
    from bpt_b200.kernels.norm_quant import rms_norm_int8

    x = rand(2, 5, 64, dtype=torch.bfloat16)
    x[1, 2] = 0.0  # an all-zero token must not divide by zero
    weight = torch.ones(64, dtype=torch.bfloat16)
    codes, scale = rms_norm_int8(x.cuda(), weight.cuda(), 1e-6)
    assert codes.shape == (2, 5, 64) and scale.shape == (2, 5, 1)
    check(codes, scale, *onq.rms_norm_int8(x, weight, 1e-6))
    assert codes[1, 2].abs().sum() == 0 and torch.isfinite(scale).all()

    wide = rand(8, 128)
    for view in (wide[:, ::2], wide[:, :64], wide[:, 1:65]):  # strided columns; rows read in place; unaligned
        codes, scale = rms_norm_int8(view.cuda(), weight.float().cuda(), 1e-6)
        check(codes, scale, *onq.rms_norm_int8(view, weight, 1e-6))

    out = (torch.empty((8, 64), dtype=torch.int8, device="cuda"), torch.empty(8, device="cuda"))
    again, s = rms_norm_int8(wide[:, :64].contiguous().cuda(), weight.float().cuda(), 1e-6, out=out, num_warps=8)
    assert again.data_ptr() == out[0].data_ptr() and s.data_ptr() == out[1].data_ptr()
    check(again, s, *onq.rms_norm_int8(wide[:, :64], weight, 1e-6))

    empty_codes, empty_scale = rms_norm_int8(torch.empty(0, 64, device="cuda"), weight.cuda(), 1e-6)
    assert empty_codes.shape == (0, 64) and empty_scale.shape == (0, 1)


@pytest.mark.parametrize("d,dtype", [(20000, torch.bfloat16), (20001, torch.bfloat16), (9000, torch.float32)])
def test_rms_norm_int8_rows_longer_than_the_registers_hold(d, dtype):
    """Past 2,048 chunks per row the remainder is read again from L2; an odd d takes the one-element path."""
    from bpt_b200.kernels.norm_quant import rms_norm_int8

    x = rand(3, d, seed=d, dtype=dtype) * 2
    weight = (rand(d, seed=1).abs() + 0.5).to(dtype)
    codes, scale = rms_norm_int8(x.cuda(), weight.cuda(), 1e-6)
    check(codes, scale, *onq.rms_norm_int8(x, weight, 1e-6))


def test_rms_norm_int8_with_the_residual_add():
    from conftest import GOLDEN

    from bpt_b200.kernels.norm_quant import rms_norm_int8

    g = torch.load(GOLDEN.with_name("norm_quant.pt"), weights_only=True)["residual"]
    h, delta = g["h"], g["delta"]
    x_out = torch.empty_like(h, device="cuda")
    codes, scale = rms_norm_int8(h.cuda(), g["weight"].cuda(), float(g["eps"]), delta=delta.cuda(), x_out=x_out)
    assert torch.equal(x_out.cpu(), h + delta)  # the model's bf16 residual tensor, bit for bit
    check(codes, scale, g["codes"], g["scale"])
    want_h, want_codes, want_scale = onq.add_rms_norm_int8(h, delta, g["weight"], float(g["eps"]))
    check(codes, scale, want_codes, want_scale)
    codes2, scale2 = rms_norm_int8(h.cuda(), g["weight"].cuda(), float(g["eps"]), delta=delta.cuda())  # no x_out
    assert torch.equal(codes2, codes) and torch.equal(scale2, scale)


def test_rms_norm_int8_rejects_bad_buffers():
    from bpt_b200.kernels.norm_quant import rms_norm_int8

    x = torch.randn(4, 64, device="cuda")
    w = torch.ones(64, device="cuda")
    with pytest.raises(ValueError):
        rms_norm_int8(x, torch.ones(63, device="cuda"), 1e-6)
    with pytest.raises(ValueError):
        rms_norm_int8(x, w, 1e-6, out=(torch.empty(4, 64, device="cuda"), torch.empty(4, device="cuda")))
    with pytest.raises(ValueError):
        rms_norm_int8(x, w, 1e-6, x_out=torch.empty_like(x))
    with pytest.raises(ValueError):
        rms_norm_int8(x.cpu(), w.cpu(), 1e-6)


@pytest.mark.parametrize("rows,d,dtype,residual", [
    (1500, 2000, torch.bfloat16, False),   # a partial last CTA; 8 chunks a lane, y kept in registers
    (1500, 500, torch.bfloat16, False),    # 500 is no multiple of 8: the one-element path
    (1100, 2048, torch.float32, False),    # 16 chunks a lane: y formed again for the codes
    (1024, 4096, torch.float16, False),    # 16 chunks a lane, 16-bit
    (20000, 256, torch.float16, False),    # more rows than resident warps: each warp loops
    (2048, 2048, torch.bfloat16, True),    # the residual add on the warp-per-row shape
    (600, 6144, torch.bfloat16, False),    # 24 chunks a lane: one CTA per SM
    (512, 8192, torch.float16, True),      # 32 chunks a lane, with the residual
    (700, 3000, torch.float32, False),     # fp32, 24 chunks of 4 a lane
])
def test_rms_norm_int8_warp_per_row_shapes(rows, d, dtype, residual):
    """From 512 rows on, a warp takes a row (persistent warps, eight rows a CTA)."""
    from bpt_b200.kernels.norm_quant import rms_norm_int8

    x = rand(rows, d, seed=rows + d, dtype=dtype) * 3
    weight = (rand(d, seed=7).abs() + 0.5).to(dtype)
    if residual:
        delta = rand(rows, d, seed=8, dtype=dtype)
        x_out = torch.empty(rows, d, dtype=dtype, device="cuda")
        codes, scale = rms_norm_int8(x.cuda(), weight.cuda(), 1e-6, delta=delta.cuda(), x_out=x_out)
        h, want_codes, want_scale = onq.add_rms_norm_int8(x, delta, weight, 1e-6)
        assert torch.equal(x_out.cpu(), h)
        check(codes, scale, want_codes, want_scale)
    else:
        codes, scale = rms_norm_int8(x.cuda(), weight.cuda(), 1e-6)
        check(codes, scale, *onq.rms_norm_int8(x, weight, 1e-6))
