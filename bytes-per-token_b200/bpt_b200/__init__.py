"""bpt_b200: fastserve's decode hot path (ish-codes-magic/bytes-per-token) as sm_100a CUDA kernels.

- `bpt_b200.kernels.w4a16`        INT4 group-wise weight-only linear (GEMV at small M), fused gate_up + SwiGLU
- `bpt_b200.kernels.kv_attention` decode attention over paged FP8 / INT8 and contiguous KIVI caches, split-K
                                  with an exact log-sum-exp merge, with the reference kernel module's signatures
- `bpt_b200.kernels.kv_write`     the quantized KV-cache write path
- `bpt_b200.workloads`            the seeded synthetic inputs of the benchmark configurations

Kernels live in libbpt_b200.so (C ABI: include/bpt_b200.h), loaded on first use through `bpt_b200._lib`.
"""

__version__ = "0.1.0"
