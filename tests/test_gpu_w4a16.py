"""W4A16 kernels against the CPU oracle (oracle/w4a16.py): codes bit-exact, bf16 outputs within
atol 1e-2 / rtol 1e-2 of the fp32 dequantize-then-matmul reference (the tolerance of the north star)."""

import pytest
import torch

from oracle import w4a16 as ow4

pytestmark = pytest.mark.gpu

TOL = {"atol": 1e-2, "rtol": 1e-2}


def dense(n, k, seed=0, std=0.02):
    return torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * std


def acts(m, k, seed=1):
    return torch.randn(m, k, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)


@pytest.mark.parametrize("n,k,group", [(6144, 2048, 128), (96, 256, 128), (64, 6144, 128), (40, 512, 64), (24, 96, 32)])
def test_quantize_is_bit_exact(n, k, group):
    from bpt_b200.kernels.w4a16 import quantize_w4a16

    w = dense(n, k, seed=n)
    w[0, :group] = 0.0  # an all-zero group
    w[1, group:] = w[1, group:].abs() + 0.01 if k > group else w[1, group:]
    for src in (w, w.to(torch.bfloat16)):
        qweight, scales, qzeros = quantize_w4a16(src.cuda(), group)
        codes, s, z = ow4.quantize_w4a16(src.float(), group)
        want_q, want_s, want_z = ow4.pack_w4a16(codes, s, z)
        assert torch.equal(qweight.cpu(), want_q)
        assert torch.equal(scales.cpu(), want_s)
        assert torch.equal(qzeros.cpu(), want_z)
        assert torch.equal(ow4.unpack_nibbles_int32(qweight.cpu(), k), codes)  # the unpacked codes, bit for bit


def check_linear(m, n, k, group, seed=0, symmetric=False, x=None):
    """The kernel against the oracle of its arithmetic: the tcgen05 GEMM multiplies with the reference model's
    dense bf16 weight (compressed.py:56-69), the others scale exact group sums in fp32."""
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_kernel, w4a16_linear

    w = dense(n, k, seed)
    x = acts(m, k, seed + 1) if x is None else x
    qweight, scales, qzeros = quantize_w4a16(w.cuda(), group)
    if symmetric:
        qzeros = None
    dense_bf16 = w4a16_kernel(m, n, k, group, zeros=qzeros is not None) == "tcgen05"
    got = w4a16_linear(x.cuda(), qweight, scales, qzeros, group=group)
    want = ow4.w4a16_linear(x, qweight.cpu(), scales.cpu(), None if qzeros is None else qzeros.cpu(), group,
                            dense_bf16=dense_bf16)
    assert got.dtype == torch.bfloat16 and got.shape == (m, n)
    torch.testing.assert_close(got.cpu().float(), want.float(), **TOL)
    # and much tighter than the tolerance against an fp64 evaluation of the same quantized weight
    codes = ow4.unpack_nibbles_int32(qweight.cpu(), k)
    zeros = None if qzeros is None else ow4.unpack_nibbles_int32(qzeros.cpu(), k // group)
    wq = ow4.dequantize_w4a16(codes, scales.cpu(), zeros, group)
    if dense_bf16:
        wq = wq.to(torch.bfloat16).float()
    exact = x.double() @ wq.double().T
    err = (got.cpu().double() - exact).abs().max().item()
    assert err <= 2 ** -8 * exact.abs().max().item() + 1e-6


def check_gate_up(got, x, fused, group=128):
    """The fused gate_up + SwiGLU output against silu(g) * u of the fp32 sums (g and u not rounded, one rounding at
    the end), the arithmetic of the kernel a shape takes, at the north star's atol / rtol 1e-2."""
    from bpt_b200.kernels.w4a16 import w4a16_kernel

    m, k = x.shape
    n = fused[0].shape[0]
    dense_bf16 = w4a16_kernel(m, n, k, group) == "tcgen05"
    want = ow4.w4a16_gate_up_silu(x, *[t.cpu() for t in fused], group, dense_bf16=dense_bf16)
    torch.testing.assert_close(got.cpu().float(), want.float(), **TOL)


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 16])
def test_linear_config1_shape(m):
    check_linear(m, 6144, 2048, 128, seed=m)


@pytest.mark.parametrize("n,k,group", [(2048, 6144, 128), (1024, 2048, 128), (12288, 2048, 128), (1000, 512, 64),
                                       (7, 96, 32), (130, 1024, 128), (33, 3072, 128)])
def test_linear_shapes(n, k, group):
    check_linear(1, n, k, group, seed=n)
    check_linear(4, n, k, group, seed=n + 1)


@pytest.mark.parametrize("m", [32, 33, 64, 100, 256])
def test_gemm_m_at_least_32(m):
    # the tiled tensor-core GEMM: M tiles of 64 (ragged last tile), N tiles of 32 (ragged: 1000, 2056)
    check_linear(m, 1000, 2048, 128, seed=m)
    check_linear(m, 2056, 6144, 128, seed=m + 1)


def test_gemm_group_64_and_symmetric():
    check_linear(64, 512, 1024, 64, seed=21)
    check_linear(48, 512, 1024, 128, seed=22, symmetric=True)


def test_gemm_gate_up_silu():
    from bpt_b200.kernels.w4a16 import interleave_rows, quantize_w4a16, w4a16_gate_up_silu

    i, k = 1536, 2048
    gate, up = dense(i, k, 13), dense(i, k, 14)
    x = acts(64, k, 15)
    qg, qu = quantize_w4a16(gate.cuda()), quantize_w4a16(up.cuda())
    fused = [interleave_rows(a, b) for a, b in zip(qg, qu, strict=True)]
    got = w4a16_gate_up_silu(x.cuda(), *fused)
    check_gate_up(got, x, fused)


def test_m16_long_k_splits_k_over_a_cluster():
    # 16 rows of x at K = 6144: the tensor-core kernel splits K over a cluster of CTAs (their x staging fits)
    check_linear(16, 256, 6144, 128, seed=11)
    check_linear(9, 264, 6144, 128, seed=12)


def test_small_n_splits_k_and_matches():
    # small N leaves SMs idle: K is split over clusters of 2-8 CTAs whose partials meet in distributed shared
    # memory (plain and fused)
    from bpt_b200.kernels.w4a16 import interleave_rows, quantize_w4a16, w4a16_gate_up_silu

    for m, n, k in [(1, 1024, 2048), (1, 256, 6144), (4, 512, 4096), (16, 128, 2048)]:
        check_linear(m, n, k, 128, seed=m + n)
    gate, up = dense(128, 2048, 31), dense(128, 2048, 32)
    x = acts(3, 2048, 33)
    qg, qu = quantize_w4a16(gate.cuda()), quantize_w4a16(up.cuda())
    fused = [interleave_rows(a, b) for a, b in zip(qg, qu, strict=True)]
    check_gate_up(w4a16_gate_up_silu(x.cuda(), *fused), x, fused)


@pytest.mark.parametrize("m,n,k,group", [(1, 16, 256, 64), (2, 4096, 2048, 32), (8, 2048, 6144, 128),
                                         (7, 512, 6144, 64), (1, 12288, 2048, 128), (3, 160, 4096, 128)])
def test_streaming_gemv_shapes(m, n, k, group):
    # M <= 8, N a multiple of 16: the persistent streaming GEMV (one tile to six tiles per CTA, ring refills,
    # groups of 32/64/128, x staging beside one stage only at K = 6144, M = 8)
    check_linear(m, n, k, group, seed=m * 7 + n)
    check_linear(m, n, k, group, seed=m * 7 + n + 1, symmetric=True)


@pytest.mark.parametrize("m,group", [(1, 128), (3, 64), (8, 128)])
def test_streaming_gemv_activation_outliers(m, group):
    # the streaming GEMV turns each (token, group) of x into integers under one power-of-two scale: a channel
    # hundreds of times larger than the rest sets that scale, so the other inputs of its group keep fewer bits
    k = 2048
    x = acts(m, k, 7).float()
    x[:, 5] = 300.0
    x[:, 700] = -1000.0
    x[0, 1500:1628] = 1e-3 * x[0, 1500:1628]  # a group of tiny values beside ordinary ones
    check_linear(m, 1024, k, group, seed=m + 90, x=x.to(torch.bfloat16))


def test_streaming_gemv_chain_under_pdl():
    # each call's weights are fetched before it waits on its predecessor; its x is the predecessor's output
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_linear

    k = 2048
    ws = [quantize_w4a16(dense(k, k, seed=40 + i).cuda()) for i in range(6)]
    x = acts(2, k, 46).cuda()
    plain, h = [], x
    for w in ws:
        h = w4a16_linear(h, *w)
        plain.append(h)
    torch.cuda.synchronize()
    outs = [torch.empty(2, k, dtype=torch.bfloat16, device="cuda") for _ in ws]
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(3):
            h = x
            for w, o in zip(ws, outs, strict=True):
                h = w4a16_linear(h, *w, out=o, pdl=True)
    torch.cuda.synchronize()
    for want, got in zip(plain, outs, strict=True):
        assert torch.equal(got, want)


def test_symmetric_layout_without_zero_points():
    check_linear(1, 512, 1024, 128, symmetric=True)


def test_config1_full_size():
    from bpt_b200 import workloads

    case = workloads.config1(keep_dense=True)
    from bpt_b200.kernels.w4a16 import w4a16_linear

    got = w4a16_linear(case.x, case.qweight, case.scales, case.qzeros, group=128)
    want = ow4.w4a16_linear(case.x.cpu(), case.qweight.cpu(), case.scales.cpu(), case.qzeros.cpu(), 128)
    torch.testing.assert_close(got.cpu().float(), want.float(), **TOL)
    assert case.bytes == 6_553_600


def test_gate_up_silu_matches_two_linears():
    from bpt_b200.kernels.w4a16 import interleave_rows, quantize_w4a16, w4a16_gate_up_silu

    i, k = 6144, 2048
    gate, up = dense(i, k, 3), dense(i, k, 4)
    for m in (1, 3, 4):
        x = acts(m, k, 5 + m)
        qg, qu = quantize_w4a16(gate.cuda()), quantize_w4a16(up.cuda())
        fused = [interleave_rows(a, b) for a, b in zip(qg, qu, strict=True)]
        check_gate_up(w4a16_gate_up_silu(x.cuda(), *fused), x, fused)


def test_out_buffer_views_and_pdl():
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_linear

    n, k = 512, 1024
    qweight, scales, qzeros = quantize_w4a16(dense(n, k).cuda())
    x = acts(6, k).cuda()
    base = w4a16_linear(x, qweight, scales, qzeros)
    out = torch.empty(6, n, dtype=torch.bfloat16, device="cuda")
    again = w4a16_linear(x, qweight, scales, qzeros, out=out, pdl=True)
    assert again.data_ptr() == out.data_ptr() and torch.equal(again, base)
    x3 = x.reshape(2, 3, k)
    assert torch.equal(w4a16_linear(x3, qweight, scales, qzeros).reshape(6, n), base)
    wide = torch.zeros(6, 2 * k, dtype=torch.bfloat16, device="cuda")
    wide[:, :k] = x
    assert torch.equal(w4a16_linear(wide[:, :k], qweight, scales, qzeros), base)  # a strided row view


def test_bad_arguments_raise_value_error():
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_linear

    qweight, scales, qzeros = quantize_w4a16(dense(64, 256).cuda())
    with pytest.raises(ValueError):
        w4a16_linear(acts(1, 256), qweight, scales, qzeros)  # activations on the CPU
    with pytest.raises(ValueError):
        w4a16_linear(acts(1, 128).cuda(), qweight, scales, qzeros)  # wrong K
    with pytest.raises(ValueError):
        w4a16_linear(acts(1, 256).cuda(), qweight, scales, qzeros, group=64)  # scales do not match the group


@pytest.mark.parametrize("m", [1, 4, 64])
def test_pack_quantized_checkpoint_serves_without_a_dense_copy(m):
    """A compressed-tensors INT4 Linear (q + 8 nibbles, bf16 group scales) loaded by from_pack_quantized runs the
    kernels on the checkpoint's own words; the result matches the reference's dense path (dequantize_linear,
    compressed.py:56-69, then nn.Linear) within the north-star tolerance."""
    from bpt_b200.kernels.w4a16 import from_pack_quantized, w4a16_kernel, w4a16_linear

    n, k = 2048, 2048
    g = torch.Generator().manual_seed(m)
    q = torch.randint(-8, 8, (n, k), generator=g)
    scale = (torch.rand(n, k // 128, generator=g) * 0.004 + 1e-3).to(torch.bfloat16)
    parts = {"weight_packed": ow4.pack_nibbles_int32((q + 8).to(torch.uint8)), "weight_scale": scale,
             "weight_shape": torch.tensor([n, k])}
    qweight, scales, qzeros, group = from_pack_quantized(parts)
    x = acts(m, k, seed=m + 1)
    got = w4a16_linear(x.cuda(), qweight.cuda(), scales.cuda(), qzeros, group=group).cpu().float()
    dense = (q.float() * scale.float().repeat_interleave(128, dim=1)).to(torch.bfloat16)  # dequantize_linear
    torch.testing.assert_close(got, torch.nn.functional.linear(x.float(), dense.float()), **TOL)
    own = ow4.w4a16_linear(x, qweight, scales, None, group, dense_bf16=w4a16_kernel(m, n, k, group, False) == "tcgen05")
    torch.testing.assert_close(got, own.float(), **TOL)


def test_unaligned_scales_take_the_cuda_core_kernel():
    """Scales that are not 16-byte aligned cannot arrive by bulk copy: the CUDA-core kernel takes the shape, with the
    same group-sum arithmetic."""
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_linear

    n, k = 512, 2048
    w = dense(n, k, 70)
    qweight, scales, qzeros = quantize_w4a16(w.cuda())
    store = torch.empty(scales.numel() + 1, dtype=torch.float16, device="cuda")
    shifted = store[1:].view_as(scales)  # 2 bytes past a 16-byte boundary
    shifted.copy_(scales)
    assert shifted.data_ptr() % 16 != 0
    for m in (1, 3):
        x = acts(m, k, 71 + m)
        got = w4a16_linear(x.cuda(), qweight, shifted, qzeros)
        want = ow4.w4a16_linear(x, qweight.cpu(), scales.cpu(), qzeros.cpu(), 128)
        torch.testing.assert_close(got.cpu().float(), want.float(), **TOL)


def test_long_k_many_rows_takes_the_mma_gemm():
    """A shape whose per-CTA scale table does not fit the tcgen05 kernel's shared memory (K = 16384 at group 64,
    enough row tiles that K is not split) goes to the mma.sync GEMM."""
    from bpt_b200.kernels.w4a16 import w4a16_kernel

    m, n, k, group = 256, 4864, 16384, 64
    assert w4a16_kernel(m, n, k, group) == "mma_gemm"
    check_linear(m, n, k, group, seed=80)
