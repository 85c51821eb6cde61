"""Config 4 at its own shapes: every Qwen3-1.7B decoder linear (q 2048->2048, k/v 2048->1024, o 2048->2048,
gate_up 2048->12288, down 6144->2048) at M in {1, 4, 16, 64, 256}, against the CPU oracle.

These are the (linear, M) pairs the benchmark sweeps, so the kernels timed there (streaming GEMV at M <= 8, the
tcgen05 GEMM with its K split over clusters and its 16-128-token tiles at M >= 16) are the ones checked here.
Tolerance: the north star's atol 1e-2 / rtol 1e-2 on bf16 outputs. The oracle follows the arithmetic of the
kernel a shape takes (`w4a16_kernel`): the tcgen05 GEMM multiplies with the dense bf16 weight round_bf16(s (q - z))
that the reference model holds after `quant/compressed.py:56-69`; the GEMV kernels scale exact fp32 group sums.
The fused gate_up + SwiGLU is compared with silu(g) * u of the fp32 sums, rounded once.
"""

import functools

import pytest
import torch

from oracle import w4a16 as ow4

pytestmark = pytest.mark.gpu

TOL = {"atol": 1e-2, "rtol": 1e-2}
LINEARS = {"q_proj": (2048, 2048), "k_proj": (1024, 2048), "v_proj": (1024, 2048), "o_proj": (2048, 2048),
           "gate_up": (12288, 2048), "down_proj": (2048, 6144)}
SWEEP_M = (1, 4, 16, 64, 256)


@functools.cache
def weight(name: str):
    """The linear's INT4 weight (quantized on the GPU), its CPU copies, and the fp32 / bf16 dense dequantized
    weights the oracle multiplies with."""
    from bpt_b200.kernels.w4a16 import quantize_w4a16

    n, k = LINEARS[name]
    w = torch.randn(n, k, generator=torch.Generator().manual_seed(n + k)) * 0.02
    qweight, scales, qzeros = quantize_w4a16(w.cuda(), 128)
    cpu = (qweight.cpu(), scales.cpu(), qzeros.cpu())
    codes = ow4.unpack_nibbles_int32(cpu[0], k)
    dense = ow4.dequantize_w4a16(codes, cpu[1], ow4.unpack_nibbles_int32(cpu[2], k // 128), 128)
    return (qweight, scales, qzeros), cpu, {False: dense, True: dense.to(torch.bfloat16).float()}


def acts(m, k, seed):
    return torch.randn(m, k, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)


@pytest.mark.parametrize("m", SWEEP_M)
@pytest.mark.parametrize("name", list(LINEARS))
def test_config4_linear_matches_oracle(name, m):
    from bpt_b200.kernels.w4a16 import w4a16_kernel, w4a16_linear

    n, k = LINEARS[name]
    gpu, _, dense = weight(name)
    x = acts(m, k, seed=m * 7 + n)
    kernel = w4a16_kernel(m, n, k, 128)
    if m >= 16:
        assert kernel == "tcgen05", kernel  # the benchmarked tensor-core path
    else:
        assert kernel == "stream", kernel  # M <= 8: the persistent streaming GEMV
    got = w4a16_linear(x.cuda(), *gpu, group=128).cpu().float()
    want = torch.nn.functional.linear(x.float(), dense[kernel == "tcgen05"]).to(torch.bfloat16).float()
    torch.testing.assert_close(got, want, **TOL)


@pytest.mark.parametrize("m", SWEEP_M)
def test_config4_gate_up_silu_matches_fp32_oracle(m):
    """The fused gate_up launch with its SwiGLU epilogue, interleaved rows, against silu(g) * u in fp32."""
    from bpt_b200.kernels.w4a16 import interleave_rows, quantize_w4a16, w4a16_gate_up_silu, w4a16_kernel

    n, k = LINEARS["gate_up"]
    g = torch.Generator().manual_seed(99)
    gate, up = torch.randn(n // 2, k, generator=g) * 0.02, torch.randn(n // 2, k, generator=g) * 0.02
    fused = [interleave_rows(a, b) for a, b in zip(quantize_w4a16(gate.cuda()), quantize_w4a16(up.cuda()), strict=True)]
    x = acts(m, k, seed=500 + m)
    got = w4a16_gate_up_silu(x.cuda(), *fused).cpu().float()
    want = ow4.w4a16_gate_up_silu(x, *[t.cpu() for t in fused], 128,
                                  dense_bf16=w4a16_kernel(m, n, k, 128) == "tcgen05").float()
    assert got.shape == (m, n // 2)
    torch.testing.assert_close(got, want, **TOL)
