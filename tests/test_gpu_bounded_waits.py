"""Every device-side wait is bounded: a wait that runs out records an error the host reads, the kernel still
finishes, and the next call on the same context is correct.

The failure is made on purpose with BPT_FLAG_TEST_STALL: the launch's first CTA stops issuing its copies partway
(every copy it did issue is still awaited, so nothing is left in flight and no GPU fault is involved), its waits for
the missing data give up after ~2 ms, the call reports device error 1 through bpt_device_error(). The outputs of
that call are undefined; the next call, without the flag, must match the oracle and report no error. For the
tcgen05 GEMM the next call also shows that the stalled CTA released its tensor memory (an allocation that a
finished CTA kept would stall every later launch on that SM).
"""

import math

import pytest
import torch

from oracle import attention as oatt
from oracle import kv_formats as okv
from oracle import w4a16 as ow4

pytestmark = pytest.mark.gpu

TEST_STALL = 0x40000000  # BPT_FLAG_TEST_STALL
ERR_TIMEOUT = 1


def test_paged_attention_wait_that_runs_out_is_reported_and_the_next_call_is_clean():
    from bpt_b200 import _lib, workloads
    from bpt_b200.kernels.kv_attention import attend, attend_workspace

    _lib.device_error()  # start from a clear flag
    lengths = [300, 1000, 40, 700]
    case = workloads.paged_case("fp8", 4, 16, 8, 128, lengths, 16, 200, seed=2, device="cuda")
    scale = 1.0 / math.sqrt(128)
    q, kv = case.q, case.kv
    b, hq, d = q.shape
    nb, bs, hkv, _ = kv.k_pool.shape
    split, n_splits = 64, -(-max(lengths) // 64)
    ws = attend_workspace(b, hq, d, n_splits, q.device)
    out = torch.empty(b, hq, d, device="cuda")
    status = _lib.lib().bpt_paged_attend(
        q.data_ptr(), _lib.dtype_code(q.dtype), q.stride(0), q.stride(1), kv.k_pool.data_ptr(), kv.v_pool.data_ptr(),
        _lib.KV_FP8, float(kv.k_scale), float(kv.v_scale), None, None, kv.block_table.data_ptr(),
        kv.block_table.stride(0), case.lengths.data_ptr(), b, hq, hkv, d, bs, nb, split, n_splits, scale,
        out.data_ptr(), _lib.DTYPE_F32, ws.data_ptr(), ws.numel(), TEST_STALL, torch.cuda.current_stream().cuda_stream)
    assert status == _lib.OK, _lib.lib().bpt_last_error()
    assert _lib.device_error() == ERR_TIMEOUT  # synchronizes: the kernel finished
    ref_kv = okv.PagedKV("fp8", kv.k_pool.cpu(), kv.v_pool.cpu(), kv.k_scale, kv.v_scale, kv.block_table.cpu(), 16)
    want = oatt.paged_attend(q.cpu(), ref_kv, case.lengths.cpu(), scale)
    for _ in range(2):  # the same workspace: the stalled call left its tickets at zero
        got = attend(q, kv, case.lengths, scale, split=split, workspace=ws)
        torch.testing.assert_close(got.cpu(), want, rtol=2e-4, atol=2e-4 * want.abs().max().item())
    assert _lib.device_error() == 0


@pytest.mark.parametrize("m,n,k", [(64, 2048, 2048), (16, 1024, 6144)])  # one CTA per tile / K split over a cluster
def test_tcgen05_wait_that_runs_out_is_reported_and_tensor_memory_is_released(m, n, k):
    from bpt_b200 import _lib
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_kernel, w4a16_linear

    assert w4a16_kernel(m, n, k) == "tcgen05"
    _lib.device_error()
    w = torch.randn(n, k, generator=torch.Generator().manual_seed(n)) * 0.02
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16)
    qweight, scales, qzeros = quantize_w4a16(w.cuda())
    xd = x.cuda()
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    status = _lib.lib().bpt_w4a16_linear(xd.data_ptr(), k, qweight.data_ptr(), scales.data_ptr(), qzeros.data_ptr(),
                                         y.data_ptr(), n, m, n, k, 128, TEST_STALL,
                                         torch.cuda.current_stream().cuda_stream)
    assert status == _lib.OK, _lib.lib().bpt_last_error()
    assert _lib.device_error() == ERR_TIMEOUT
    want = ow4.w4a16_linear(x, qweight.cpu(), scales.cpu(), qzeros.cpu(), 128, dense_bf16=True)
    for _ in range(3):  # every SM's tensor memory is free again: these launches allocate it and finish
        got = w4a16_linear(xd, qweight, scales, qzeros)
        torch.testing.assert_close(got.cpu().float(), want.float(), atol=1e-2, rtol=1e-2)
    assert _lib.device_error() == 0
