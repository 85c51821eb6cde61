"""bpt_paged_attend_noalloc, the paged decode attention entry point that allocates nothing.

It exists for callers that cannot allocate device memory — an engine that gave all free HBM to its paged KV pool
at start-up, a runtime that forbids device allocation after initialization, a foreign-language host that only
holds the buffers it was handed — so its split partials live in a fixed static device array instead of a
caller workspace. This test calls it through the C ABI and checks that two calls in a row give the output of
the workspace entry point (bpt_paged_attend, through `attend`) within the attention tolerance the other tests
use, and that a request larger than the fixed array is refused before anything launches.

The file name sorts last so that, in a run that stops at the first failure, every other test has already run.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def call_noalloc(case, scale, split, n_splits, out):
    from bpt_b200 import _lib

    kv = case.kv
    if kv.kind == "fp8":
        code, ks, vs, kss, vss = _lib.KV_FP8, float(kv.k_scale), float(kv.v_scale), None, None
    else:
        code, ks, vs, kss, vss = _lib.KV_INT8, 1.0, 1.0, kv.k_scale.data_ptr(), kv.v_scale.data_ptr()
    q = case.q
    b, hq, d = q.shape
    nb, bs, hkv, _ = kv.k_pool.shape
    return _lib.lib().bpt_paged_attend_noalloc(
        q.data_ptr(), _lib.dtype_code(q.dtype), q.stride(0), q.stride(1), kv.k_pool.data_ptr(), kv.v_pool.data_ptr(),
        code, ks, vs, kss, vss, kv.block_table.data_ptr(), kv.block_table.stride(0), case.lengths.data_ptr(), b, hq,
        hkv, d, bs, nb, split, n_splits, scale, out.data_ptr(), _lib.dtype_code(out.dtype), 0,
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("kind", ["fp8", "int8"])
def test_no_alloc_attend_matches_the_workspace_entry_point_on_two_calls(kind):
    from bpt_b200 import _lib, workloads
    from bpt_b200.kernels.kv_attention import attend

    lengths = [700, 1, 300, 0, 129]
    case = workloads.paged_case(kind, 5, 16, 8, 128, lengths, 16, 96, seed=21, device="cuda")
    scale = 1.0 / math.sqrt(128)
    split, tokens = 64, max(lengths)
    n_splits = -(-tokens // split)
    want = attend(case.q, case.kv, case.lengths, scale, split=split, tokens=tokens)
    tol = 2e-4 * want.abs().max().item()
    for _ in range(2):  # the second call finds what the first left in the shared array
        out = torch.full_like(want, float("nan"))
        status = call_noalloc(case, scale, split, n_splits, out)
        assert status == _lib.OK, _lib.lib().bpt_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out, want, rtol=2e-4, atol=tol)
        assert out[3].abs().sum() == 0  # the empty sequence
    bf = torch.empty(5, 16, 128, dtype=torch.bfloat16, device="cuda")
    assert call_noalloc(case, scale, split, n_splits, bf) == _lib.OK
    torch.testing.assert_close(bf.float(), want, atol=1e-2, rtol=1e-2)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("variant", ["16 KV heads", "strided q"])
def test_no_alloc_split_kernel_branch_matches_on_two_calls(variant):
    """Shapes the persistent kernel does not take (more than 8 KV heads; q rows with a head stride other than D)
    run the split kernels with per-sequence tickets: the same two-call check against the workspace entry point."""
    import dataclasses

    from bpt_b200 import _lib, workloads
    from bpt_b200.kernels.kv_attention import attend

    lengths = [500, 3, 260]
    hkv = 16 if variant == "16 KV heads" else 8
    case = workloads.paged_case("fp8", 3, 16, hkv, 128, lengths, 16, 64, seed=31, device="cuda")
    if variant == "strided q":
        wide = torch.zeros(3, 16, 256, dtype=case.q.dtype, device="cuda")
        wide[..., :128] = case.q
        case = dataclasses.replace(case, q=wide[..., :128])
        assert case.q.stride(1) == 256
    scale = 1.0 / math.sqrt(128)
    split, tokens = 64, max(lengths)
    want = attend(case.q, case.kv, case.lengths, scale, split=split, tokens=tokens)
    for _ in range(2):
        out = torch.full_like(want, float("nan"))
        assert call_noalloc(case, scale, split, -(-tokens // split), out) == _lib.OK, _lib.lib().bpt_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out, want, rtol=2e-4, atol=2e-4 * want.abs().max().item())
    assert _lib.device_error() == 0


def test_no_alloc_refuses_tensors_of_another_device_than_the_current_one():
    """The array used is the current device's: host memory passed as q is refused before anything launches."""
    from bpt_b200 import _lib, workloads

    case = workloads.paged_case("fp8", 2, 16, 8, 128, [40, 17], 16, 8, seed=4, device="cuda")
    host_q = case.q.cpu().pin_memory()
    import dataclasses

    out = torch.zeros(2, 16, 128, device="cuda")
    status = call_noalloc(dataclasses.replace(case, q=host_q), 0.1, 16, 3, out)
    assert status == _lib.ERR_INVALID
    assert out.abs().sum() == 0


def test_no_alloc_refuses_a_request_beyond_its_fixed_scratch():
    from bpt_b200 import _lib, workloads

    # 2,100 one-token sequences: at least 2,100 partials of 16 heads x 129 floats, above the 16 MiB array
    b = 2100
    case = workloads.paged_case("fp8", b, 16, 8, 128, [1] * b, 16, b, seed=3, device="cuda")
    out = torch.zeros(b, 16, 128, device="cuda")
    status = call_noalloc(case, 0.1, 16, 1, out)
    assert status == _lib.ERR_WORKSPACE
    assert b"scratch" in _lib.lib().bpt_last_error()
    assert out.abs().sum() == 0  # nothing was launched
