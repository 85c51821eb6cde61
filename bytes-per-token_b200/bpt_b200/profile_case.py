"""Run one hot-path kernel a few times on one workload, for profilers (ncu) and quick timing.

    python -m bpt_b200.profile_case attention-config2 [--launches 4]
    python -m bpt_b200.profile_case attention-config3
    python -m bpt_b200.profile_case gemv-config1

Each case builds its seeded synthetic inputs once, then launches the kernel `--launches` times back to back and
prints the mean device time per launch (CUDA events; not a benchmark number under a profiler).
"""

from __future__ import annotations

import argparse
import math

import torch

from . import workloads
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
    ap.add_argument("case", choices=["attention-config2", "attention-config3", "gemv-config1"])
    ap.add_argument("--launches", type=int, default=4)
    args = ap.parse_args()
    if args.case == "gemv-config1":
        us = _gemv(args.launches)
    else:
        us = _attention(2 if args.case.endswith("2") else 3, args.launches)
    print(f"{args.case}: {us:.1f} us per launch (mean of {args.launches}, after one warm-up launch)")


if __name__ == "__main__":
    main()
