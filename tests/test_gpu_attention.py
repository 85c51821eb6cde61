"""Paged FP8 / INT8 decode attention and the split merge against the CPU oracle (oracle/attention.py), the
KV write path bit for bit against oracle/kv_formats.py.

Attention tolerance: the reference's own kernel check, rtol 2e-4 and atol 2e-4 * max|want|
(tests/kernels/test_kernels_gpu.py:84), for fp32 outputs; bf16 outputs within atol 1e-2 / rtol 1e-2.
"""

import math

import pytest
import torch

from oracle import attention as oatt
from oracle import kv_formats as okv

pytestmark = pytest.mark.gpu


def close(got, want):
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got, want, rtol=2e-4, atol=2e-4 * max(want.abs().max().item(), 1e-6))


def to_oracle(kv):
    """The GPU pool as the oracle's PagedKV (CPU copies)."""
    ks = kv.k_scale if kv.kind == "fp8" else kv.k_scale.cpu()
    vs = kv.v_scale if kv.kind == "fp8" else kv.v_scale.cpu()
    return okv.PagedKV(kv.kind, kv.k_pool.cpu(), kv.v_pool.cpu(), ks, vs, kv.block_table.cpu(), kv.block_size)


def small_case(kind, batch, q_heads, kv_heads, d, lengths, seed=0, num_blocks=None):
    from bpt_b200 import workloads

    pages = sum(-(-n // 16) for n in lengths)
    return workloads.paged_case(kind, batch, q_heads, kv_heads, d, list(lengths), 16, num_blocks or max(pages + 7, 8),
                                seed, "cuda")


CASES = [
    # batch, Hq, Hkv, D, lengths
    (4, 16, 8, 128, [160, 1, 70, 0]),
    (3, 16, 8, 128, [16, 17, 33]),
    (2, 8, 8, 128, [300, 129]),
    (2, 32, 8, 128, [64, 200]),
    (2, 64, 8, 128, [48, 97]),
    (2, 4, 2, 64, [100, 31]),
    (2, 8, 4, 256, [90, 240]),
    (1, 16, 8, 128, [4096]),
]


@pytest.mark.parametrize("kind", ["fp8", "int8"])
@pytest.mark.parametrize("batch,hq,hkv,d,lengths", CASES)
def test_paged_partials_match_oracle(kind, batch, hq, hkv, d, lengths):
    from bpt_b200.kernels.kv_attention import decode_attention

    case = small_case(kind, batch, hq, hkv, d, lengths, seed=len(lengths) + d)
    scale = 1 / math.sqrt(d)
    tokens = max(lengths)
    okv_ = to_oracle(case.kv)
    for split in (16, 64, max(16, -(-tokens // 16) * 16)):
        out, lse = decode_attention(case.q, case.kv, case.lengths, scale, tokens=tokens, split=split)
        want_out, want_lse = oatt.paged_decode_partials(case.q.cpu(), okv_, case.lengths.cpu(), scale, split, tokens)
        assert out.shape == want_out.shape and lse.shape == want_lse.shape
        close(out.cpu(), want_out)
        finite = torch.isfinite(want_lse)
        assert torch.equal(torch.isfinite(lse.cpu()), finite)  # empty splits: -inf exactly where the oracle has it
        torch.testing.assert_close(lse.cpu()[finite], want_lse[finite], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("kind", ["fp8", "int8"])
@pytest.mark.parametrize("batch,hq,hkv,d,lengths", CASES)
def test_paged_attend_fused_merge_matches_oracle(kind, batch, hq, hkv, d, lengths):
    from bpt_b200.kernels.kv_attention import attend

    case = small_case(kind, batch, hq, hkv, d, lengths, seed=7 + d)
    scale = 1 / math.sqrt(d)
    want = oatt.paged_attend(case.q.cpu(), to_oracle(case.kv), case.lengths.cpu(), scale)
    for split in (16, 32, None):
        got = attend(case.q, case.kv, case.lengths, scale, split=split)
        close(got.cpu(), want)
        got2 = attend(case.q, case.kv, case.lengths, scale, split=split)  # counters were left at zero
        assert torch.equal(got, got2)
    bf = torch.empty(batch, hq, d, dtype=torch.bfloat16, device="cuda")
    attend(case.q, case.kv, case.lengths, scale, out=bf, split=32)
    torch.testing.assert_close(bf.cpu().float(), want, atol=1e-2, rtol=1e-2)
    if 0 in lengths:
        assert bf[lengths.index(0)].abs().sum() == 0  # no tokens: zeros, not NaN


@pytest.mark.parametrize("kind", ["fp8", "int8"])
@pytest.mark.parametrize("batch,hq,hkv,d,lengths", [CASES[0], CASES[1], (3, 16, 8, 128, [5000, 0, 2049])])
def test_early_start_under_pdl_matches_plain(kind, batch, hq, hkv, d, lengths):
    # kv_ready: pages are mapped and copied before the wait on the previous kernel (q, out and the workspace
    # after it); a chain of such calls (the previous one writing the same out and workspace) equals plain calls,
    # with empty sequences, pages that all fit the first stages, and long sequences that refill the stages
    from bpt_b200.kernels.kv_attention import attend

    case = small_case(kind, batch, hq, hkv, d, lengths, seed=3 + d)
    scale = 1 / math.sqrt(d)
    want = attend(case.q, case.kv, case.lengths, scale)
    other = small_case(kind, batch, hq, hkv, d, lengths, seed=99)
    out = torch.full((batch, hq, d), float("nan"), device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(3):
            attend(other.q, other.kv, other.lengths, scale, out=out, pdl=True, kv_ready=True)
            attend(case.q, case.kv, case.lengths, scale, out=out, pdl=True, kv_ready=True)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    close(out.cpu(), oatt.paged_attend(case.q.cpu(), to_oracle(case.kv), case.lengths.cpu(), scale))


def test_config2_full_size_against_oracle():
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_attention import attend

    case = workloads.config2()
    scale = 1 / math.sqrt(128)
    got = attend(case.q, case.kv, case.lengths, scale, tokens=4096)
    want = oatt.paged_attend(case.q.cpu(), to_oracle(case.kv), case.lengths.cpu(), scale)
    close(got.cpu(), want)
    bf = attend(case.q, case.kv, case.lengths, scale, tokens=4096, out=torch.empty_like(case.q))
    torch.testing.assert_close(bf.cpu().float(), want, atol=1e-2, rtol=1e-2)


def test_config3_long_context_int8_split_invariance_and_oracle_row():
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_attention import PagedQuantKV, attend

    case = workloads.config3()
    scale = 1 / math.sqrt(128)
    got = attend(case.q, case.kv, case.lengths, scale, tokens=32768)
    # the merge is exact: any split gives the same attention
    for split in (2048, 32768):
        close(attend(case.q, case.kv, case.lengths, scale, tokens=32768, split=split), got)
    # and one sequence against the oracle (the CPU holds one row of 32,768 tokens comfortably)
    kv = case.kv
    row = PagedQuantKV(kv.kind, kv.k_pool, kv.v_pool, kv.block_table[:1], kv.block_size, kv.k_scale, kv.v_scale)
    want = oatt.paged_attend(case.q[:1].cpu(), to_oracle(row), case.lengths[:1].cpu(), scale)
    close(got[:1].cpu(), want)


def test_merge_partials_kernel_matches_oracle():
    from bpt_b200.kernels.kv_attention import merge_partials

    g = torch.Generator().manual_seed(3)
    outs = torch.randn(3, 4, 5, 64, generator=g)
    lses = torch.randn(3, 4, 5, generator=g) * 4
    lses[1, :, 2] = -math.inf  # an empty split
    lses[2] = -math.inf  # a row with no tokens at all
    outs[2] = 0.0
    got = merge_partials(outs.cuda(), lses.cuda())
    want = oatt.merge_partials(outs, lses)
    torch.testing.assert_close(got.cpu(), want, rtol=1e-5, atol=1e-6)
    assert got[2].abs().sum() == 0
    into = torch.full((3, 4, 64), float("nan"), dtype=torch.bfloat16, device="cuda")
    assert merge_partials(outs.cuda(), lses.cuda(), out=into).data_ptr() == into.data_ptr()
    torch.testing.assert_close(into.cpu().float(), want, rtol=1e-2, atol=1e-2)  # written in out's own dtype
    # many splits per row (a CTA per row spreads them over its threads)
    outs = torch.randn(2, 16, 300, 128, generator=g)
    lses = torch.randn(2, 16, 300, generator=g) * 4
    torch.testing.assert_close(merge_partials(outs.cuda(), lses.cuda()).cpu(), oatt.merge_partials(outs, lses),
                               rtol=1e-5, atol=1e-6)


def test_out_of_range_block_entry_is_recorded_not_read():
    """The kernel bounds-checks every block-table entry before it addresses the pool."""
    from bpt_b200 import _lib
    from bpt_b200.kernels.kv_attention import attend

    case = small_case("fp8", 2, 16, 8, 128, [40, 20], seed=1)
    _lib.device_error()  # clear
    bad = case.kv.block_table.clone()
    bad[0, 1] = case.kv.num_blocks + 5
    case.kv.block_table = bad
    got = attend(case.q, case.kv, case.lengths, 1 / math.sqrt(128))
    assert _lib.device_error() == 2
    assert torch.isfinite(got).all()
    assert _lib.device_error() == 0  # reading clears it


# ---- the write path ---------------------------------------------------------------------------------------------


@pytest.mark.parametrize("kind", ["fp8", "int8"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("d", [64, 128, 256])
def test_paged_write_is_bit_exact(kind, dtype, d):
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_write import quantize_kv_paged

    b, hkv, q, bs, nb = 3, 4, 5, 16, 12
    g = torch.Generator().manual_seed(d)
    table = torch.randperm(nb, generator=g)[: b * 2].reshape(b, 2).to(torch.int32)
    kv = workloads.empty_pool(kind, nb, bs, hkv, d, "cuda", table.cuda(), scale=0.05)
    k = (torch.randn(b, hkv, q, d, generator=g) * 3).to(dtype)
    v = (torch.randn(b, hkv, q, d, generator=g) * 3).to(dtype)
    k[0, 0, 0] = 0.0  # an all-zero vector
    k[1, 1, 1, :4] = torch.tensor([1000.0, -1000.0, 20.0, -20.0]).to(dtype)  # saturates in FP8
    pos = torch.tensor([[0, 1, 2, 3, 4], [14, 15, 16, 17, 18], [5, 9, 20, 30, 31]])
    blocks = torch.gather(table.long(), 1, pos // bs)
    offsets = pos % bs
    quantize_kv_paged(k.cuda(), v.cuda(), kv, blocks.cuda(), offsets.cuda())
    want = to_oracle(workloads.empty_pool(kind, nb, bs, hkv, d, "cuda", table.cuda(), scale=0.05))
    okv.paged_write(want, k, v, blocks, offsets)
    assert torch.equal(kv.k_pool.cpu(), want.k_pool) and torch.equal(kv.v_pool.cpu(), want.v_pool)
    if kind == "int8":
        assert torch.equal(kv.k_scale.cpu(), want.k_scale) and torch.equal(kv.v_scale.cpu(), want.v_scale)


@pytest.mark.parametrize("kind", ["fp8", "int8"])
@pytest.mark.parametrize("q,d", [(1, 128), (4, 64), (19, 128), (9, 256)])
def test_paged_write_many_tokens_is_bit_exact(kind, q, d):
    # from 4 new tokens on, a warp writes up to 8 consecutive tokens of one head (19: groups of 8, 8 and 3), each to
    # its own scattered slot, eight values per lane; a decode step's single token keeps one warp per token
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_write import quantize_kv_paged

    b, hkv, bs, nb = 3, 8, 16, 12
    g = torch.Generator().manual_seed(5)
    table = torch.randperm(nb, generator=g)[: b * 2].reshape(b, 2).to(torch.int32)
    kv = workloads.empty_pool(kind, nb, bs, hkv, d, "cuda", table.cuda(), scale=0.05)
    k = (torch.randn(b, hkv, q, d, generator=g) * 3).to(torch.bfloat16)
    v = (torch.randn(b, hkv, q, d, generator=g) * 3).to(torch.bfloat16)
    pos = torch.stack([torch.randperm(2 * bs, generator=g)[:q] for _ in range(b)])
    blocks = torch.gather(table.long(), 1, pos // bs)
    offsets = pos % bs
    quantize_kv_paged(k.cuda(), v.cuda(), kv, blocks.cuda(), offsets.cuda())
    want = to_oracle(workloads.empty_pool(kind, nb, bs, hkv, d, "cuda", table.cuda(), scale=0.05))
    okv.paged_write(want, k, v, blocks, offsets)
    assert torch.equal(kv.k_pool.cpu(), want.k_pool) and torch.equal(kv.v_pool.cpu(), want.v_pool)
    if kind == "int8":
        assert torch.equal(kv.k_scale.cpu(), want.k_scale) and torch.equal(kv.v_scale.cpu(), want.v_scale)


@pytest.mark.parametrize("q", [2, 12])
def test_paged_write_out_of_range_slot_is_recorded_and_skipped(q):
    # one token's write block lies outside the pool and another's offset outside its block: both are recorded on the
    # device and written nowhere, every other token is written as usual (one warp per token at 2 tokens, warps of 8
    # tokens at 12)
    from bpt_b200 import _lib, workloads
    from bpt_b200.kernels.kv_write import quantize_kv_paged

    b, hkv, d, bs, nb = 2, 8, 128, 16, 8
    table = torch.arange(4, dtype=torch.int32).reshape(b, 2)
    kv = workloads.empty_pool("int8", nb, bs, hkv, d, "cuda", table.cuda())
    g = torch.Generator().manual_seed(q)
    k = torch.randn(b, hkv, q, d, generator=g).to(torch.bfloat16)
    pos = torch.arange(q).expand(b, q)
    blocks = torch.gather(table.long(), 1, pos // bs).clone()
    offsets = (pos % bs).clone()
    blocks[0, 1] = nb + 3
    offsets[1, q - 1] = bs
    _lib.device_error()  # clear
    quantize_kv_paged(k.cuda(), k.cuda(), kv, blocks.cuda(), offsets.cuda())
    assert _lib.device_error() in (2, 3)
    keep = torch.ones(b, q, dtype=torch.bool)
    keep[0, 1] = keep[1, q - 1] = False
    want = to_oracle(workloads.empty_pool("int8", nb, bs, hkv, d, "cuda", table.cuda()))
    okv.paged_write(want, k[:, :, :1], k[:, :, :1], blocks[:, :1], offsets[:, :1])  # tokens 0 of both sequences
    for j in range(1, q):
        rows = [i for i in range(b) if keep[i, j]]
        if rows:
            okv.paged_write(want, k[rows][:, :, j:j + 1], k[rows][:, :, j:j + 1], blocks[rows][:, j:j + 1],
                            offsets[rows][:, j:j + 1])
    assert torch.equal(kv.k_pool.cpu(), want.k_pool) and torch.equal(kv.k_scale.cpu(), want.k_scale)


@pytest.mark.parametrize("q", [1, 12])
def test_paged_fp8_write_keeps_the_sign_of_zero(q):
    # x / scale of a -0 input is -0, whose E4M3 code is 0x80 (the reference's cast), not 0x00
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_write import quantize_kv_paged

    b, hkv, d, bs, nb = 2, 8, 128, 16, 4
    table = torch.arange(4, dtype=torch.int32).reshape(b, 2)
    kv = workloads.empty_pool("fp8", nb, bs, hkv, d, "cuda", table.cuda(), scale=0.05)
    k = torch.randn(b, hkv, q, d, generator=torch.Generator().manual_seed(q)).to(torch.bfloat16)
    k[:, :, :, ::3] = -0.0
    k[:, :, :, 1::5] = 0.0
    pos = torch.arange(q).expand(b, q)
    blocks, offsets = torch.gather(table.long(), 1, pos // bs), pos % bs
    quantize_kv_paged(k.cuda(), k.cuda(), kv, blocks.cuda(), offsets.cuda())
    want = to_oracle(workloads.empty_pool("fp8", nb, bs, hkv, d, "cuda", table.cuda(), scale=0.05))
    okv.paged_write(want, k, k, blocks, offsets)
    assert (want.k_pool == 0x80).any()
    assert torch.equal(kv.k_pool.cpu(), want.k_pool) and torch.equal(kv.v_pool.cpu(), want.v_pool)


def test_paged_write_from_a_transposed_view():
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_write import quantize_kv_paged

    b, hkv, q, d = 2, 8, 3, 128
    table = torch.arange(4, dtype=torch.int32).reshape(2, 2)
    kv = workloads.empty_pool("int8", 4, 16, hkv, d, "cuda", table.cuda())
    base = torch.randn(b, q, hkv, d, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    k = base.cuda().transpose(1, 2)  # [B, Hkv, Q, D] view of a [B, Q, Hkv, D] projection output
    pos = torch.arange(q).expand(b, q)
    quantize_kv_paged(k, k, kv, torch.gather(table.long(), 1, pos // 16).cuda(), (pos % 16).cuda())
    want = to_oracle(workloads.empty_pool("int8", 4, 16, hkv, d, "cuda", table.cuda()))
    okv.paged_write(want, base.transpose(1, 2), base.transpose(1, 2), torch.gather(table.long(), 1, pos // 16), pos % 16)
    assert torch.equal(kv.k_pool.cpu(), want.k_pool) and torch.equal(kv.k_scale.cpu(), want.k_scale)
