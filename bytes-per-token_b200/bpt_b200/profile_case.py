"""Run one hot-path kernel a few times on one workload, for profilers (ncu) and quick timing.

    python -m bpt_b200.profile_case attention-config2 [--launches 4]
    python -m bpt_b200.profile_case attention-config3
    python -m bpt_b200.profile_case gemv-config1
    python -m bpt_b200.profile_case w4a16-sweep
    python -m bpt_b200.profile_case gate-up-m64      (gate-up-m256)
    python -m bpt_b200.profile_case norm-quant       (one [16384, 2048] bf16 rms_norm_int8 per launch)
    python -m bpt_b200.profile_case norm-quant-sweep
    python -m bpt_b200.profile_case kivi-sweep       (contiguous KIVI decode attention, bits 4 / 8 / 16)
    python -m bpt_b200.profile_case kv-write-sweep   (paged FP8 / INT8 cache writes, KIVI group quantize)

Each kernel case builds its seeded synthetic inputs once, then launches the kernel `--launches` times back to
back and prints the mean device time per launch (CUDA events; not a benchmark number under a profiler).
`w4a16-sweep` is config 4: every Qwen3-1.7B decoder linear at M in {1, 4, 16, 64, 256}, each timed by replaying
a CUDA graph of calls that rotate over enough weight copies to exceed L2 (so every call reads HBM), with
programmatic dependent launch; it prints a markdown table of us per call, GB/s (algorithmic bytes) and TFLOP/s.
`norm-quant-sweep` times rms_norm_int8 (RMSNorm + per-token INT8) the same way over rotating inputs.
"""

from __future__ import annotations

import argparse
import math

import torch

from . import workloads
from .workloads import w4a16_bytes
from .kernels.kv_attention import attend, attend_workspace
from .kernels.w4a16 import quantize_w4a16, w4a16_linear


def _attention(config: int, launches: int) -> float:
    case = workloads.config2() if config == 2 else workloads.config3()
    b, hq, d = case.q.shape
    tokens = case.max_length
    out = torch.empty(b, hq, d, dtype=torch.float32, device=case.q.device)
    ws = attend_workspace(b, hq, d, -(-tokens // 256), case.q.device)
    run = lambda: attend(case.q, case.kv, case.lengths, 1.0 / math.sqrt(d), out=out, workspace=ws)
    return _time(run, launches)


def _gemv(launches: int) -> float:
    g = torch.Generator(device="cuda").manual_seed(0)
    w = torch.randn(6144, 2048, generator=g, device="cuda") * 0.02
    qw, sc, qz = quantize_w4a16(w, 128)
    x = torch.randn(1, 2048, generator=g, device="cuda").to(torch.bfloat16)
    y = torch.empty(1, 6144, dtype=torch.bfloat16, device="cuda")
    return _time(lambda: w4a16_linear(x, qw, sc, qz, out=y), launches)


SWEEP_SHAPES = [("q_proj / o_proj", 2048, 2048), ("k_proj / v_proj", 1024, 2048), ("gate_up (fused, SiLU)", 12288, 2048),
                ("down_proj", 2048, 6144)]
SWEEP_M = [1, 4, 16, 64, 256]


def _sweep() -> None:
    from .kernels.w4a16 import w4a16_gate_up_silu

    peak = _peak_gbs()
    print("| linear | N x K | M | us per call | GB/s | of HBM peak | TFLOP/s |")
    print("|---|---|---|---|---|---|---|")
    for name, n, k in SWEEP_SHAPES:
        copies = max(2, min(40, int(300e6 // (n * k // 2))))
        g = torch.Generator(device="cuda").manual_seed(n + k)
        ws = [quantize_w4a16(torch.randn(n, k, generator=g, device="cuda") * 0.02, 128) for _ in range(copies)]
        fused = name.startswith("gate_up")
        for m in SWEEP_M:
            x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
            y = torch.empty(m, n // 2 if fused else n, dtype=torch.bfloat16, device="cuda")
            fn = w4a16_gate_up_silu if fused else w4a16_linear
            stream = torch.cuda.Stream()
            with torch.cuda.stream(stream):
                for w in ws:
                    fn(x, *w, out=y, pdl=True)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for w in ws:
                    fn(x, *w, out=y, pdl=True)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 10
            start.record()
            for _ in range(reps):
                graph.replay()
            end.record()
            torch.cuda.synchronize()
            us = start.elapsed_time(end) * 1e3 / (reps * copies)
            nbytes = w4a16_bytes(m, n, k) - (2 * m * n // 2 if fused else 0)
            gbs = nbytes / us / 1e3
            print(f"| {name} | {n} x {k} | {m} | {us:.2f} | {gbs:.0f} | {gbs / peak:.1%} | {2 * m * n * k / us / 1e6:.1f} |",
                  flush=True)
            del graph
        del ws
        torch.cuda.empty_cache()


NORM_SHAPES = [(64, 2048, False), (64, 2048, True), (256, 2048, False), (4096, 2048, False), (16384, 2048, False),
               (16384, 2048, True), (16384, 6144, False)]


def norm_quant_bytes(rows: int, d: int, residual: bool, esize: int = 2) -> int:
    """x read, codes and scales written, the weight once; with the residual also delta read and x + delta written."""
    return rows * d * (esize + 1) + rows * 4 + d * esize + (2 * rows * d * esize if residual else 0)


def _norm_quant(launches: int) -> float:
    from .kernels.norm_quant import rms_norm_int8

    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(16384, 2048, generator=g, device="cuda") * 3).to(torch.bfloat16)
    w = (torch.rand(2048, generator=g, device="cuda") + 0.5).to(torch.bfloat16)
    out = (torch.empty(16384, 2048, dtype=torch.int8, device="cuda"), torch.empty(16384, device="cuda"))
    return _time(lambda: rms_norm_int8(x, w, 1e-6, out=out), launches)


def _norm_quant_sweep() -> None:
    from .kernels.norm_quant import rms_norm_int8

    peak = _peak_gbs()
    print("| rows x d (bf16) | residual | us per call | GB/s | of HBM peak |")
    print("|---|---|---|---|---|")
    for rows, d, residual in NORM_SHAPES:
        nbytes = norm_quant_bytes(rows, d, residual)
        copies = max(2, min(40, int(300e6 // nbytes)))
        g = torch.Generator(device="cuda").manual_seed(rows + d)
        xs = [(torch.randn(rows, d, generator=g, device="cuda") * 3).to(torch.bfloat16) for _ in range(copies)]
        ds = [torch.randn(rows, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(copies)] if residual else None
        w = (torch.rand(d, generator=g, device="cuda") + 0.5).to(torch.bfloat16)
        outs = [(torch.empty(rows, d, dtype=torch.int8, device="cuda"), torch.empty(rows, device="cuda"))
                for _ in range(copies)]
        sums = [torch.empty_like(xs[0]) for _ in range(copies)] if residual else None

        def calls():
            for i in range(copies):
                if residual:
                    rms_norm_int8(xs[i], w, 1e-6, out=outs[i], delta=ds[i], x_out=sums[i], pdl=True)
                else:
                    rms_norm_int8(xs[i], w, 1e-6, out=outs[i], pdl=True)

        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            calls()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            calls()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        start.record()
        for _ in range(reps):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
        us = start.elapsed_time(end) * 1e3 / (reps * copies)
        gbs = nbytes / us / 1e3
        print(f"| {rows} x {d} | {'yes' if residual else 'no'} | {us:.2f} | {gbs:.0f} | {gbs / peak:.1%} |", flush=True)
        del graph, xs, ds, outs, sums
        torch.cuda.empty_cache()


def _graph_us(calls, copies: int, reps: int = 10) -> float:
    """us per call of `calls()` (which makes `copies` calls), replayed as one CUDA graph after warm-up."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        calls()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        calls()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    us = start.elapsed_time(end) * 1e3 / (reps * copies)
    del graph
    return us


def kivi_bytes(batch: int, kv_heads: int, tokens: int, head_dim: int, bits: int, group: int = 32) -> int:
    """K and V codes, the keys' per-channel grids (fp16 scale + zero per group of tokens), the values' per-token
    grids, for every token of every sequence and KV head (q and the output are negligible)."""
    if bits == 16:
        return batch * kv_heads * tokens * head_dim * 2 * 2
    codes = head_dim // 2 if bits == 4 else head_dim
    return batch * kv_heads * tokens * (2 * codes + 2 * 2 * head_dim // group + 2 * 2)


def _kivi_sweep() -> None:
    """The contiguous KIVI path (`attend` over a QuantKV: split kernel + merge kernel) on the reference's quoted
    case, one 32k-token sequence with 16 Q / 8 KV heads and D 128, and on a batch of 8 such sequences."""
    from .kernels.kv_write import quantize_kv

    peak = _peak_gbs()
    print("| batch x tokens | bits | us per call | GB/s | of HBM peak |")
    print("|---|---|---|---|---|")
    hq, hkv, d, t = 16, 8, 128, 32768
    for batch in (1, 8):
        for bits in (4, 8, 16):
            nbytes = kivi_bytes(batch, hkv, t, d, bits)
            copies = max(2, min(8, int(400e6 // nbytes)))
            g = torch.Generator(device="cuda").manual_seed(batch * 100 + bits)
            caches = []
            for _ in range(copies):
                k = torch.randn(batch, hkv, t, d, generator=g, device="cuda").to(torch.bfloat16)
                v = torch.randn(batch, hkv, t, d, generator=g, device="cuda").to(torch.bfloat16)
                caches.append(quantize_kv(k, v, bits))
                del k, v
            q = torch.randn(batch, hq, d, generator=g, device="cuda").to(torch.bfloat16)
            lengths = torch.full((batch,), t, dtype=torch.int32, device="cuda")
            out = torch.empty(batch, hq, d, device="cuda")

            def calls():
                for kv in caches:
                    attend(q, kv, lengths, 1.0 / math.sqrt(d), out=out, tokens=t)

            us = _graph_us(calls, copies)
            gbs = nbytes / us / 1e3
            print(f"| {batch} x {t} | {bits} | {us:.2f} | {gbs:.0f} | {gbs / peak:.1%} |", flush=True)
            del caches
            torch.cuda.empty_cache()


def _kv_write_sweep() -> None:
    """The paged cache write (quantize_kv_paged: FP8 per-tensor scale, INT8 per (token, head) fp16 scale) for one
    decode token per sequence and for 512-token blocks, and the KIVI group quantize (quantize_kv_into)."""
    from .kernels.kv_write import empty_quant_kv, quantize_kv_into, quantize_kv_paged

    peak = _peak_gbs()
    print("| write | shape (B x Hkv x tokens x D, bf16 in) | us per call | GB/s | of HBM peak |")
    print("|---|---|---|---|---|")
    hkv, d, bs = 8, 128, 16
    for kind in ("fp8", "int8"):
        for batch, q in ((64, 1), (32, 512)):
            elems = batch * hkv * q * d
            nbytes = 2 * elems * 2 + 2 * elems + (2 * batch * hkv * q * 2 if kind == "int8" else 0) + 2 * batch * q * 4
            copies = max(2, min(40, int(300e6 // nbytes)))
            g = torch.Generator(device="cuda").manual_seed(batch + q)
            blocks = batch * q // bs + batch
            kvs = [workloads.empty_pool(kind, blocks, bs, hkv, d, "cuda", None) for _ in range(copies)]
            ks = [torch.randn(batch, hkv, q, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(copies)]
            vs = [torch.randn(batch, hkv, q, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(copies)]
            slot = torch.arange(batch * q, device="cuda", dtype=torch.int32).view(batch, q)
            wb, wo = (slot // bs).contiguous(), (slot % bs).contiguous()

            def calls():
                for i in range(copies):
                    quantize_kv_paged(ks[i], vs[i], kvs[i], wb, wo)

            us = _graph_us(calls, copies)
            gbs = nbytes / us / 1e3
            print(f"| paged {kind} | {batch} x {hkv} x {q} x {d} | {us:.2f} | {gbs:.0f} | {gbs / peak:.1%} |", flush=True)
            del kvs, ks, vs
            torch.cuda.empty_cache()
    for bits in (4, 8):
        batch, t = 8, 4096
        elems = batch * hkv * t * d
        nbytes = 2 * elems * 2 + kivi_bytes(batch, hkv, t, d, bits)
        copies = 2
        g = torch.Generator(device="cuda").manual_seed(bits)
        ks = [torch.randn(batch, hkv, t, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(copies)]
        vs = [torch.randn(batch, hkv, t, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(copies)]
        caches = [empty_quant_kv(batch, hkv, t, d, bits, 32, "cuda") for _ in range(copies)]

        def calls():
            for i in range(copies):
                quantize_kv_into(ks[i], vs[i], caches[i], 0)

        us = _graph_us(calls, copies)
        gbs = nbytes / us / 1e3
        print(f"| KIVI {bits}-bit quantize | {batch} x {hkv} x {t} x {d} | {us:.2f} | {gbs:.0f} | {gbs / peak:.1%} |",
              flush=True)
        del ks, vs, caches
        torch.cuda.empty_cache()


def _gate_up(m: int, launches: int) -> float:
    """The fused gate_up linear of config 4 (12288 x 2048) at M tokens: one weight copy."""
    from .kernels.w4a16 import w4a16_gate_up_silu

    g = torch.Generator(device="cuda").manual_seed(0)
    qw, sc, qz = quantize_w4a16(torch.randn(12288, 2048, generator=g, device="cuda") * 0.02, 128)
    x = torch.randn(m, 2048, generator=g, device="cuda").to(torch.bfloat16)
    y = torch.empty(m, 6144, dtype=torch.bfloat16, device="cuda")
    return _time(lambda: w4a16_gate_up_silu(x, qw, sc, qz, out=y), launches)


def _peak_gbs() -> float:
    import json
    from pathlib import Path

    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    return float(json.loads(path.read_text())["hbm_gbs"]) if path.exists() else 6650.0


def _time(fn, launches: int) -> float:
    fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(launches):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) * 1e3 / launches


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=["attention-config2", "attention-config3", "gemv-config1", "w4a16-sweep",
                                     "gate-up-m64", "gate-up-m256", "norm-quant", "norm-quant-sweep", "kivi-sweep",
                                     "kv-write-sweep"])
    ap.add_argument("--launches", type=int, default=4)
    args = ap.parse_args()
    if args.case == "w4a16-sweep":
        _sweep()
        return
    if args.case == "norm-quant-sweep":
        _norm_quant_sweep()
        return
    if args.case == "kivi-sweep":
        _kivi_sweep()
        return
    if args.case == "kv-write-sweep":
        _kv_write_sweep()
        return
    if args.case == "norm-quant":
        us = _norm_quant(args.launches)
    elif args.case == "gemv-config1":
        us = _gemv(args.launches)
    elif args.case.startswith("gate-up-m"):
        us = _gate_up(int(args.case.split("-m")[1]), args.launches)
    else:
        us = _attention(2 if args.case.endswith("2") else 3, args.launches)
    print(f"{args.case}: {us:.1f} us per launch (mean of {args.launches}, after one warm-up launch)")


if __name__ == "__main__":
    main()
