"""Run one hot-path kernel a few times on one workload, for profilers (ncu) and quick timing.

    python -m bpt_b200.profile_case attention-config2 [--launches 4]
    python -m bpt_b200.profile_case attention-config3
    python -m bpt_b200.profile_case gemv-config1
    python -m bpt_b200.profile_case w4a16-sweep
    python -m bpt_b200.profile_case gate-up-m64      (gate-up-m256)
    python -m bpt_b200.profile_case norm-quant       (one [16384, 2048] bf16 rms_norm_int8 per launch)
    python -m bpt_b200.profile_case norm-quant-sweep

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
                                     "gate-up-m64", "gate-up-m256", "norm-quant", "norm-quant-sweep"])
    ap.add_argument("--launches", type=int, default=4)
    args = ap.parse_args()
    if args.case == "w4a16-sweep":
        _sweep()
        return
    if args.case == "norm-quant-sweep":
        _norm_quant_sweep()
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
