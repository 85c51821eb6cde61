"""CPU oracle for the decode hot path: TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU, the reference's own arithmetic for the three parts of
fastserve's decode hot path (ish-codes-magic/bytes-per-token, `src/fastserve/...`):

- `oracle.w4a16`      asymmetric INT4 group-wise weights: grid, codes, int32 nibble packing, dequantize, linear
- `oracle.kv_formats` the quantized KV formats: FP8 E4M3 with a per-tensor scale, symmetric INT8 with an fp16
                      scale per (token, head), and the KIVI contiguous grids with nibble packing
- `oracle.attention`  partial attention with its log-sum-exp, the exact merge of splits, the paged gather,
                      and the unfused decode attention (gather, dequantize, attend) for paged and KIVI caches

Every function names the reference file:line it follows. The restatement is pinned against golden vectors
produced by the reference itself (`tests/golden/make_golden.py` imports the reference and writes
`tests/golden/golden.pt`) and against the known-answer values of the reference's own tests.

Who may use it: only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py`, and there
only as the checker or as the timed CPU baseline. The product package (`bytes-per-token_b200/bpt_b200`) never
imports it: its kernels run on the GPU or raise.
"""
