"""Host-side logic that needs no GPU: argument checks that raise before any launch, split heuristics, the
synthetic workloads' byte accounting and block tables."""

import pytest
import torch


def test_kernels_refuse_cpu_tensors():
    from bpt_b200.kernels.kv_attention import PagedQuantKV, attend, decode_attention, merge_partials
    from bpt_b200.kernels.kv_write import quantize_kv_paged
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_linear

    with pytest.raises(ValueError, match="no CPU path"):
        quantize_w4a16(torch.zeros(8, 128))
    with pytest.raises(ValueError, match="no CPU path"):
        w4a16_linear(torch.zeros(1, 128, dtype=torch.bfloat16), torch.zeros(8, 16, dtype=torch.int32),
                     torch.zeros(8, 1, dtype=torch.float16))
    kv = PagedQuantKV("fp8", torch.zeros(2, 16, 1, 64, dtype=torch.uint8), torch.zeros(2, 16, 1, 64, dtype=torch.uint8),
                      torch.zeros(1, 2, dtype=torch.int32), 16)
    q = torch.zeros(1, 1, 64)
    lengths = torch.ones(1, dtype=torch.int32)
    for fn in (decode_attention, attend):
        with pytest.raises(ValueError, match="no CPU path"):
            fn(q, kv, lengths, 0.125)
    with pytest.raises(ValueError, match="no CPU path"):
        merge_partials(torch.zeros(1, 1, 1, 4), torch.zeros(1, 1, 1))
    with pytest.raises(ValueError, match="no CPU path"):
        quantize_kv_paged(torch.zeros(1, 1, 1, 64), torch.zeros(1, 1, 1, 64), kv, torch.zeros(1, 1), torch.zeros(1, 1))


def test_default_split_is_the_reference_rule():
    """tests/kernels/test_kernels_gpu.py:136-142 of the reference, which runs only on a GPU there."""
    from bpt_b200.kernels.kv_attention import default_split

    assert default_split(1, 8, 32768) == 128
    assert default_split(64, 8, 8192) == 256
    assert default_split(1, 8, 100) == 128
    assert all(default_split(b, 8, t) % 32 == 0 for b in (1, 3, 64) for t in (1, 1000, 30000))


def test_paged_split_is_a_power_of_two_page_multiple():
    from bpt_b200.kernels.kv_attention import paged_split

    for b, t in [(32, 4096), (8, 32768), (1, 100), (64, 8192), (1, 32768), (256, 16)]:
        s = paged_split(b, t)
        assert s % 16 == 0 and s & (s - 1) == 0 and 64 <= s <= 1024
    assert paged_split(1, 32768) < paged_split(64, 32768)  # one long sequence gets more splits


def test_byte_accounting_matches_the_configs():
    from bpt_b200.workloads import paged_bytes, w4a16_bytes

    assert w4a16_bytes(1, 6144, 2048) == 6_553_600  # config 1: codes + scales + zeros + x + y
    assert w4a16_bytes(256, 6144, 2048) == 10_731_520
    assert w4a16_bytes(1, 12288, 2048) == 13_103_104
    lengths = torch.full((8,), 32768)
    kv = 8 * 32768 * 2080
    table = 4 * 8 * 2048
    assert paged_bytes(lengths, 16, 8, 128, "int8") == kv + table + 2 * 8 * 16 * 128 * 2  # config 3
    assert paged_bytes(torch.tensor([16]), 16, 8, 128, "fp8") == 16 * 2048 + 4 + 2 * 16 * 128 * 2


def test_block_tables_draw_distinct_pages():
    from bpt_b200.workloads import block_table_for

    g = torch.Generator().manual_seed(0)
    lengths = torch.randint(512, 4097, (32,), generator=g)
    table = block_table_for(lengths, 16, 16384, g)
    used = torch.cat([table[i, : (int(n) + 15) // 16] for i, n in enumerate(lengths)])
    assert used.unique().numel() == used.numel()  # no page shared between or within sequences
    assert int(table.min()) >= 0 and int(table.max()) < 16384
    with pytest.raises(ValueError, match="pages needed"):
        block_table_for(torch.tensor([17]), 16, 1, g)
