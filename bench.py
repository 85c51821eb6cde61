"""Benchmark of fastserve's decode hot path on B200: W4A16 GEMV (config 1) + paged FP8-KV decode attention
(config 2), one step = one GEMV and one attention over one batch, inputs resident in HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU; weak scaling, no collective)
    python bench.py --case NAME [--launches L]             (one kernel on one workload, for ncu; or a sweep table)

Prints one JSON line (rank 0). `value` is whole-job achieved HBM bandwidth: the algorithmic bytes of every
rank's steps over the slowest rank's device time. `e2e` is the same metric through the public Python API with
this step's inputs copied from pinned host memory and the results copied back inside the timed region (one
staging copy each way: the kernels read and write views of one device buffer per direction).
`--impl reference` times the reference's CPU path (the oracle port: dequantize-then-matmul and gather,
dequantize, attend) on the host cores, over the same workload (the whole config-2 batch and the config-1 GEMV).

Inputs larger than L2: the GEMV rotates over 40 weight copies (262 MB) and the attention over 3 batches with
their own pools (about 450 MB of KV touched per cycle), so no step finds its data in the 126 MB L2.

`kernels.*` adds, each in its own device-timed region: config 3 (INT8 32k-token attention), the config-4 sweep
(every Qwen3-1.7B decoder linear at M in {1, 4, 16, 64, 256}), the next row past the path (RMSNorm + per-token
INT8 of [16384, 2048] bf16 rows) and, on more than one GPU, the column-parallel W4A16 linear (NCCL all-gather).
`decode_step` is config 5 (the Qwen3-1.7B decode step, batch 64 per GPU, one CUDA graph per step).
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT, ROOT / "bytes-per-token_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import torch  # noqa: E402

METRIC = "achieved HBM GB/s (% of B200 peak) and us/call: W4A16 GEMV + FP8-KV decode attn"
WORKLOAD = ("config1 W4A16 GEMV (M=1, K=2048, N=6144, asym INT4 g128) + config2 paged FP8 decode attention "
            "(B=32, 16 Q / 8 KV heads, D=128, lengths U[512,4096], page 16, 16384-page pool)")
GEMV_COPIES = 40
ATTN_BATCHES = 3
E2E_GROUP = 6  # steps per wait of the kernels' stream on the copy stream in the end-to-end region
CONFIG3_BATCHES = 2  # 2 x 545 MB of INT8 KV
NQ_ROWS, NQ_D, NQ_COPIES = 16384, 2048, 3  # rms_norm_int8: 3 x 64 MB of bf16 rows rotate (above L2)
SWEEP_LINEARS = [("q_proj", 2048, 2048), ("k_proj", 1024, 2048), ("v_proj", 1024, 2048), ("o_proj", 2048, 2048),
                 ("gate_up", 12288, 2048), ("down_proj", 2048, 6144)]
SWEEP_M = (1, 4, 16, 64, 256)
SWEEP_BYTES = 160e6  # weight copies per linear: at least this many bytes, so the rotation exceeds L2
PROFILE_SUMMARY = ROOT / "profiles" / "paged_attention_fp8_config2.md"


def norm_quant_bytes(rows: int, d: int, residual: bool) -> int:
    """rms_norm_int8's algorithmic bytes: bf16 x read, int8 codes and fp32 scales written, the weight once; with the
    residual also delta read and x + delta written."""
    return rows * d * 3 + rows * 4 + d * 2 + (4 * rows * d if residual else 0)


def measured_peaks() -> dict:
    """HBM GB/s and dense bf16 TFLOP/s (sustained) from MEASURED_PEAKS.json, else the recipe's fallback."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        m = json.loads(path.read_text())
        return {"hbm_gbs": float(m["hbm_gbs"]), "tflops": float(m.get("bf16_tflops_sustained", 1400.0)),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "tflops": 1400.0, "source": "fallback"}


def profiled_traffic() -> tuple[int, int] | None:
    """(DRAM bytes, algorithmic bytes) per launch of the attention kernel from the committed ncu summary (lines
    `traffic_bytes_per_launch: N` and `algorithmic_bytes_per_launch: N`, both averaged over the captured launches)."""
    if not PROFILE_SUMMARY.exists():
        return None
    found = {}
    for line in PROFILE_SUMMARY.read_text().splitlines():
        key, _, val = line.strip().partition(":")
        if key in ("traffic_bytes_per_launch", "algorithmic_bytes_per_launch"):
            found[key] = int(val.strip().replace(",", ""))
    if len(found) != 2:
        return None
    return found["traffic_bytes_per_launch"], found["algorithmic_bytes_per_launch"]


# ---- clocks -----------------------------------------------------------------------------------------------------


class ClockSampler:
    """Samples this GPU's SM clock and throttle reasons through NVML every ~2 ms in a background thread."""

    REASONS = {
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
        "sw_power_cap": 0x4,
    }

    def __init__(self, device: torch.device):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nvml = pynvml
        except Exception as exc:  # no NVML: report no clocks rather than fail the run
            self._nvml = None
            self.error = repr(exc)

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = statistics.median(s[0] for s in self.samples)
        seen = 0
        for _, r in self.samples:
            seen |= r
        reasons = [name for name, bit in self.REASONS.items() if seen & bit]
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples)}


# ---- ranks --------------------------------------------------------------------------------------------------------


def gather_ranks(local: dict, dist) -> list[dict]:
    """Every rank's measurement dict, in rank order, on every rank (one all_gather_object; None: one process)."""
    if dist is None:
        return [local]
    gathered = [None] * dist.get_world_size()
    dist.all_gather_object(gathered, local)
    return gathered


def combine_ranks(gathered: list[dict]) -> dict:
    """Whole-job figures: the slowest rank's device time for each timed region, the sum of every rank's bytes
    (and decode tokens). Each rank runs the same number of steps on its own batch (weak scaling)."""
    out = {
        "total_ms": max(g["total_ms"] for g in gathered),
        "e2e_ms": max(g["e2e_ms"] for g in gathered),
        "bytes": sum(g["bytes"] for g in gathered),
    }
    if all("decode_ms" in g for g in gathered):
        out["decode_ms"] = max(g["decode_ms"] for g in gathered)
        out["decode_tokens"] = sum(g["decode_tokens"] for g in gathered)
        out["decode_bytes"] = sum(g["decode_bytes"] for g in gathered)
    return out


def per_rank_record(gathered: list[dict], steps: int, decode_steps: int) -> list[dict]:
    """Each rank's own figures, so a straggler can be named: step and decode-step device times, the host's enqueue
    time per step, and the rank's median SM clock."""
    rows = []
    for r, g in enumerate(gathered):
        row = {"rank": r, "step_ms": round(g["total_ms"] / steps, 5),
               "host_enqueue_ms": round(g.get("host_step_ms", 0.0), 4), "sm_mhz": g["clocks"]["sm_mhz"]}
        if "decode_ms" in g:
            row["decode_step_ms"] = round(g["decode_ms"] / decode_steps, 4)
        rows.append(row)
    return rows


# ---- device timing ------------------------------------------------------------------------------------------------


class Timer:
    """Device time of K calls of a function (ms): CUDA events on the launching stream around the whole sequence,
    with the GPU asleep before the region while the host enqueues the launches (so the events time kernels, not
    Python launch overhead), barrier + synchronize on both sides."""

    def __init__(self, device, dist):
        self.device, self.dist = device, dist
        self.clock_khz = torch.cuda.get_device_properties(device).clock_rate or 2_000_000

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()
        torch.cuda.synchronize(self.device)

    def host_seconds(self, fn, calls: int = 8) -> float:
        """Host time to enqueue one call (after a synchronize)."""
        self.barrier()
        t0 = time.perf_counter()
        for i in range(calls):
            fn(i)
        s = (time.perf_counter() - t0) / calls
        self.barrier()
        return s

    def __call__(self, fn, steps: int, host_s: float | None = None) -> float:
        host_s = self.host_seconds(fn) if host_s is None else host_s
        lead = int(min(0.5, 2.0 * host_s * steps + 1e-3) * self.clock_khz * 1e3)
        stream = torch.cuda.current_stream(self.device)
        self.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(lead)
        start.record(stream)
        for k in range(steps):
            fn(k)
        end.record(stream)
        self.barrier()
        return start.elapsed_time(end)


# ---- our arm ------------------------------------------------------------------------------------------------------


def build_inputs(device: torch.device, seed: int, attention: bool = True):
    from bpt_b200 import workloads
    from bpt_b200.kernels.w4a16 import quantize_w4a16

    g = torch.Generator(device=device).manual_seed(seed)
    weights = []
    for _ in range(GEMV_COPIES):
        w = torch.randn(6144, 2048, generator=g, device=device) * 0.02
        weights.append(quantize_w4a16(w, 128))
    x = torch.randn(1, 2048, generator=g, device=device).to(torch.bfloat16)
    # every rank draws the same lengths (batch i's from seed i, as rank 0 builds them) with its own queries, table and
    # pool, so the per-GPU work is the same at every N (weak scaling) and the slowest rank is not merely the busiest
    attn = ([workloads.config2(device=device, seed=seed * 100 + i, lengths_seed=i) for i in range(ATTN_BATCHES)]
            if attention else [])
    return weights, x, attn


def run_ours(args, rank: int, world: int, device: torch.device) -> dict | None:
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_attention import attend, attend_workspace, paged_split
    from bpt_b200.kernels.w4a16 import w4a16_linear

    dist = torch.distributed if world > 1 else None
    timer = Timer(device, dist)
    weights, x, attn = build_inputs(device, seed=rank)
    scale = 1.0 / math.sqrt(128)
    y = torch.empty(1, 6144, dtype=torch.bfloat16, device=device)
    out = torch.empty(32, 16, 128, dtype=torch.bfloat16, device=device)
    split = paged_split(32, 4096, 16, torch.cuda.get_device_properties(device).multi_processor_count)
    n_splits = -(-4096 // split)
    attend_workspace(32, 16, 128, n_splits, device)  # allocated before timing
    gemv_bytes = workloads.w4a16_bytes(1, 6144, 2048)
    attn_bytes = [c.bytes for c in attn]

    def gemv(i: int):
        qw, sc, qz = weights[i % GEMV_COPIES]
        w4a16_linear(x, qw, sc, qz, out=y, pdl=True)

    def attention(i: int):
        case = attn[i % ATTN_BATCHES]
        # kv_ready: the preceding kernel (the GEMV, or the previous attention call) writes none of this call's
        # lengths, block table or pools, so the kernel maps and copies its first pages before waiting on it
        attend(case.q, case.kv, case.lengths, scale, out=out, tokens=4096, split=split, pdl=True, kv_ready=True)

    def step(i: int):
        gemv(i)
        attention(i)

    for i in range(max(args.warmup, 3)):
        step(i)
    host_step_s = timer.host_seconds(step)

    # device-timed regions: the step (the metric), then each kernel alone (the per-kernel rooflines)
    sampler = ClockSampler(device)
    with sampler:
        soak_end = time.perf_counter() + 0.3  # the sampler needs a few hundred ms of the same load around the region
        i = 0
        while time.perf_counter() < soak_end:
            step(i)
            i += 1
            if i % 64 == 0:
                torch.cuda.synchronize(device)
        total_ms = timer(step, args.steps, host_step_s)
        attn_total_ms = timer(attention, args.steps)
        gemv_total_ms = timer(gemv, args.steps)
    local = {"total_ms": total_ms, "host_step_ms": host_step_s * 1e3, "bytes": sum(
        gemv_bytes + attn_bytes[k % ATTN_BATCHES] for k in range(args.steps)),
             "gemv_ms": gemv_total_ms / args.steps, "attn_ms": attn_total_ms / args.steps,
             "clocks": sampler.summary()}
    local["e2e_ms"], local["h2d"], local["d2h"] = e2e_timing(args, device, timer, weights, x, attn, scale, split)
    del weights, attn
    torch.cuda.empty_cache()

    kernels = {}
    if not args.quick:
        kernels["paged_attention_int8_config3"] = config3_timing(args, rank, device, timer)
        kernels["w4a16_sweep_config4"] = sweep_timing(args, rank, device, timer)
        kernels["rms_norm_int8"] = norm_quant_timing(args, rank, device, timer)
    if world > 1:
        kernels["column_parallel_w4a16"] = column_parallel_timing(args, world, device, timer)
    local["kernels"] = kernels
    if not args.no_decode:
        local.update(decode_step_timing(args, rank, device, timer))
    gathered = gather_ranks(local, dist)
    if rank != 0:
        return None
    return report(args, world, gathered, gemv_bytes, attn_bytes, split)


def report(args, world: int, gathered: list[dict], gemv_bytes: int, attn_bytes: list[int], split: int) -> dict:
    whole = combine_ranks(gathered)
    t_max, e_max, all_bytes = whole["total_ms"], whole["e2e_ms"], whole["bytes"]
    gbs = all_bytes / (t_max * 1e-3) / 1e9
    e2e_gbs = all_bytes / (e_max * 1e-3) / 1e9
    peaks = measured_peaks()
    peak = peaks["hbm_gbs"]
    r0 = gathered[0]
    attn_bytes_avg = statistics.fmean(attn_bytes)
    achieved = attn_bytes_avg / (r0["attn_ms"] * 1e-3) / 1e9
    prof = profiled_traffic()
    # the committed capture's DRAM bytes per launch, scaled to this run's batches by their algorithmic bytes (the
    # kernel reads each visible page once, so its traffic follows its algorithmic bytes)
    traffic = None if prof is None else round(prof[0] * attn_bytes_avg / prof[1])
    clocks = r0["clocks"]
    reasons = sorted({r for g in gathered for r in g["clocks"]["reasons"]})
    kernels = {
        "w4a16_gemv": {"us_per_call": round(r0["gemv_ms"] * 1e3, 2),
                       "gbs": round(gemv_bytes / (r0["gemv_ms"] * 1e-3) / 1e9, 1),
                       "frac_of_peak": round(gemv_bytes / (r0["gemv_ms"] * 1e-3) / 1e9 / peak, 3), "bytes": gemv_bytes,
                       "timing": "a chain of calls over 40 rotating weight copies, each waiting on its predecessor "
                                 "(programmatic dependent launch)"},
        "paged_attention_fp8": {"us_per_call": round(r0["attn_ms"] * 1e3, 2), "gbs": round(achieved, 1),
                                "frac_of_peak": round(achieved / peak, 3), "bytes": round(attn_bytes_avg)},
    }
    kernels.update(r0["kernels"])
    line = {
        "metric": METRIC,
        "value": round(gbs, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_max / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; random INT4 weights N(0,0.02), K/V N(0,1) in E4M3, bf16 queries N(0,1))",
        "config": {
            "workload": WORKLOAD,
            "per_rank": "one GEMV + one attention over a batch of 32 sequences per step",
            "l2": f"inputs larger than L2: {GEMV_COPIES} rotating weight copies, {ATTN_BATCHES} rotating batches/pools",
            "timing": "device lead: the host enqueues the K steps while the GPU sleeps before the region",
            "launch": "programmatic dependent launch: each kernel's prologue overlaps the previous kernel's tail",
            "split": split,
            "parallelism": f"dp{world} (independent request batches, no collective)",
        },
        "kernels": kernels,
        "roofline": {
            "kernel": "paged_attn_persistent_kernel<128, 2, FP8> (fused split merge)",
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "peak_source": f"{peaks['source']} hbm_gbs",
            "unit": "GB/s",
            "frac": round(achieved / peak, 3),
            "traffic": traffic,
            "traffic_source": None if prof is None else
            f"ncu dram bytes of {PROFILE_SUMMARY.relative_to(ROOT)} ({prof[0]} per launch over {prof[1]} algorithmic), "
            "scaled to this run's batches by algorithmic bytes",
        },
        "e2e": {"value": round(e2e_gbs, 1), "unit": "GB/s", "h2d_bytes_per_step": r0["h2d"],
                "d2h_bytes_per_step": r0["d2h"], "ms_per_step": round(e_max / args.steps, 5),
                "copies": "every step's inputs host->device (one copy per step) and results device->host (one copy "
                          "per step, as soon as the step is done), pinned buffers, on a copy stream beside the "
                          f"kernels; inputs cross a group of {E2E_GROUP} steps ahead and the kernels' stream waits "
                          "on the copy stream once per group"},
        "gpu_launches": 2 * args.steps,
        "gpu_launches_note": "the step region; the per-kernel regions launch K more of each kernel",
        "clocks": {"sm_mhz": clocks["sm_mhz"], "sm_max_mhz": clocks["sm_max_mhz"], "reasons": reasons,
                   "samples": clocks["samples"], "window": "0.3 s soak of the same step + the timed region"},
        "per_rank": per_rank_record(gathered, args.steps, args.decode_steps),
    }
    if "decode_ms" in whole:
        ms = whole["decode_ms"] / args.decode_steps
        line["decode_step"] = {
            "config": "config 5: Qwen3-1.7B decode step (28 layers, hidden 2048, intermediate 6144, 16 Q / 8 KV heads, "
                      "head_dim 128), random INT4 g128 weights + FP8 KV, batch 64 per GPU, contexts U[1024,8192]; "
                      "one CUDA graph per step; independent batches per rank, no collective",
            "tokens_per_s": round(whole["decode_tokens"] / (whole["decode_ms"] * 1e-3), 1),
            "ms_per_step": round(ms, 4),
            "gbs": round(whole["decode_bytes"] / (whole["decode_ms"] * 1e-3) / 1e9, 1),
            "bytes_per_step_per_gpu": r0["decode_bytes"] // args.decode_steps,
            "steps": args.decode_steps,
            "scaling": "weak",
        }
    if world == 1:
        line["cpu_baseline"] = cpu_baseline(repeats=3)
        if "rms_norm_int8" in line["kernels"]:
            line["kernels"]["rms_norm_int8"]["cpu_baseline"] = norm_quant_cpu_baseline()
    return line


def e2e_timing(args, device, timer, weights, x, attn, scale, split):
    """The same step through the public API with host buffers: a step's inputs (x, q, lengths, block table) sit in
    one pinned buffer and cross in one copy into one device buffer that the kernels read through views; the two
    results (y, out) are views of one device buffer and come back in one copy. As a serving loop with a prefetch queue
    does, the copies run on a copy stream beside the kernels, a group of E2E_GROUP steps at a time (the first group a
    single step): the next group's inputs cross (one copy per step) while this group computes, and each step's results
    come back as soon as the step is done. The kernels' stream waits on the copy stream once per group (the group's inputs have landed, the output
    buffers it reuses have been read back), not between every two steps: a wait there would also cut the
    programmatic dependent launch between one step's attention and the next step's GEMV. Every step's two copies lie
    inside the timed region, which the copy stream's last result closes. Returns (ms, h2d, d2h bytes)."""
    from bpt_b200.kernels.kv_attention import attend
    from bpt_b200.kernels.w4a16 import w4a16_linear

    def layout(parts):  # [(name, bytes)] -> ({name: offset}, total), each part 256-byte aligned
        offs, at = {}, 0
        for name, nb in parts:
            offs[name] = at
            at += (nb + 255) // 256 * 256
        return offs, at

    def view(buf, off, like):
        return buf[off: off + like.numel() * like.element_size()].view(like.dtype).view(like.shape)

    nb, grp = ATTN_BATCHES, E2E_GROUP
    ring = 2 * grp  # device input and output buffers: a group being computed and the next one crossing
    assert ring % nb == 0  # buffer r always holds batch r mod nb
    y = torch.empty(1, 6144, dtype=torch.bfloat16, device=device)
    out = torch.empty(32, 16, 128, dtype=torch.bfloat16, device=device)
    stage_in, pin_in, cases = [], [], []
    for r in range(ring):  # each batch its own layout (block-table widths differ)
        c = attn[r % nb]
        ioff, in_total = layout([("x", x.numel() * 2), ("q", c.q.numel() * 2), ("lengths", c.lengths.numel() * 4),
                                 ("table", c.kv.block_table.numel() * 4)])
        dev = torch.empty(in_total, dtype=torch.uint8, device=device)
        xv, qv, lv, tv = (view(dev, ioff["x"], x), view(dev, ioff["q"], c.q), view(dev, ioff["lengths"], c.lengths),
                          view(dev, ioff["table"], c.kv.block_table))
        xv.copy_(x), qv.copy_(c.q), lv.copy_(c.lengths), tv.copy_(c.kv.block_table)
        stage_in.append(dev)
        if r < nb:
            pin_in.append(dev.cpu().pin_memory())
        cases.append((xv, qv, lv, dataclasses.replace(c.kv, block_table=tv)))
    ooff, out_total = layout([("y", y.numel() * 2), ("out", out.numel() * 2)])
    stage_out = [torch.empty(out_total, dtype=torch.uint8, device=device) for _ in range(ring)]
    out_views = [(view(b, ooff["y"], y), view(b, ooff["out"], out)) for b in stage_out]
    pin_out = [torch.empty(out_total, dtype=torch.uint8).pin_memory() for _ in range(ring)]
    # the bytes that cross per step (padding included), averaged over the rotating batches
    h2d, d2h = round(sum(t.numel() for t in stage_in[:nb]) / nb), out_total

    comp = torch.cuda.current_stream(device)
    copy = torch.cuda.Stream(device)

    def run(steps: int, lead_cycles: int):
        # groups of steps [bounds[g], bounds[g + 1]): the first holds one step, so the kernels start after one
        # step's inputs have crossed, not a whole group's
        bounds = [0] + list(range(1, steps, grp)) + [steps]
        groups = len(bounds) - 1
        in_ready = [None] * groups  # the group's input copies have landed
        done = [None] * steps       # step i's kernels are done (its input and output buffers are read / filled)
        read = [None] * steps       # step i's results have been copied back
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if lead_cycles:
            torch.cuda._sleep(lead_cycles)  # the GPU waits while the host enqueues the steps
        start.record(comp)
        copy.wait_event(start)

        def h2d_group(g: int):
            with torch.cuda.stream(copy):
                last_user = bounds[g + 1] - 1 - ring  # the latest earlier step on one of the group's buffers
                if last_user >= 0:
                    copy.wait_event(done[last_user])
                for i in range(bounds[g], bounds[g + 1]):
                    stage_in[i % ring].copy_(pin_in[i % nb], non_blocking=True)
                in_ready[g] = torch.cuda.Event()
                in_ready[g].record(copy)

        h2d_group(0)
        for g in range(groups):
            if g + 1 < groups:
                h2d_group(g + 1)
            comp.wait_event(in_ready[g])
            last_user = bounds[g + 1] - 1 - ring  # its output buffers were last filled by steps up to this one
            if last_user >= 0:
                comp.wait_event(read[last_user])
            for i in range(bounds[g], bounds[g + 1]):
                xv, qv, lv, kv = cases[i % ring]
                qw, sc, qz = weights[i % GEMV_COPIES]
                y_v, out_v = out_views[i % ring]
                w4a16_linear(xv, qw, sc, qz, out=y_v, pdl=True)
                attend(qv, kv, lv, scale, out=out_v, tokens=4096, split=split, pdl=True, kv_ready=True)
                done[i] = torch.cuda.Event()
                done[i].record(comp)
                with torch.cuda.stream(copy):
                    copy.wait_event(done[i])
                    pin_out[i % ring].copy_(stage_out[i % ring], non_blocking=True)
                    read[i] = torch.cuda.Event()
                    read[i].record(copy)
        comp.wait_event(read[steps - 1])
        end.record(comp)
        return start, end

    run(3, 0)
    timer.barrier()
    t0 = time.perf_counter()
    run(3, 0)
    host_s = (time.perf_counter() - t0) / 3
    timer.barrier()
    lead = int(min(0.5, 2.0 * host_s * args.steps + 1e-3) * timer.clock_khz * 1e3)
    start, end = run(args.steps, lead)
    timer.barrier()
    return start.elapsed_time(end), h2d, d2h


def config3_timing(args, rank: int, device, timer) -> dict:
    """Config 3: INT8 KV (fp16 scale per token and KV head), 8 x 32,768 tokens, split-K with the fused merge;
    calls rotate over CONFIG3_BATCHES batches with their own pools."""
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_attention import attend

    cases = [workloads.config3(device=device, seed=rank * 100 + 50 + i) for i in range(CONFIG3_BATCHES)]
    out = torch.empty(8, 16, 128, dtype=torch.bfloat16, device=device)
    scale = 1.0 / math.sqrt(128)

    def call(i):
        c = cases[i % CONFIG3_BATCHES]
        attend(c.q, c.kv, c.lengths, scale, out=out, tokens=32768, pdl=True, kv_ready=True)

    for i in range(3):
        call(i)
    ms = timer(call, args.steps) / args.steps
    nbytes = statistics.fmean(c.bytes for c in cases)
    peak = measured_peaks()["hbm_gbs"]
    del cases
    torch.cuda.empty_cache()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"us_per_call": round(ms * 1e3, 2), "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 3),
            "bytes": round(nbytes), "workload": "B=8 x 32768 tokens, 16 Q / 8 KV heads, D 128, symmetric INT8 + fp16 "
            f"scale per (token, head), page 16, {CONFIG3_BATCHES} rotating batches"}


def sweep_timing(args, rank: int, device, timer) -> list[dict]:
    """Config 4: every Qwen3-1.7B decoder linear (gate_up fused with SwiGLU) at M in SWEEP_M; each pair a chain of K
    calls over enough weight copies to exceed L2, programmatic dependent launch. `frac_of_roofline` is the ideal
    time max(bytes / HBM peak, flops / sustained bf16 peak) over the measured time."""
    from bpt_b200 import workloads
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_gate_up_silu, w4a16_kernel, w4a16_linear

    peaks = measured_peaks()
    rows = []
    for name, n, k in SWEEP_LINEARS:
        copies = max(2, min(160, math.ceil(SWEEP_BYTES / (n * k // 2))))
        g = torch.Generator(device=device).manual_seed(1000 * rank + n + k)
        ws = [quantize_w4a16(torch.randn(n, k, generator=g, device=device) * 0.02, 128) for _ in range(copies)]
        fused = name == "gate_up"
        fn = w4a16_gate_up_silu if fused else w4a16_linear
        for m in SWEEP_M:
            x = torch.randn(m, k, generator=g, device=device).to(torch.bfloat16)
            y = torch.empty(m, n // 2 if fused else n, dtype=torch.bfloat16, device=device)

            def call(i, x=x, y=y):
                fn(x, *ws[i % copies], out=y, pdl=True)

            for i in range(3):
                call(i)
            steps = max(args.steps, 2 * copies)  # every copy at least twice
            us = timer(call, steps) / steps * 1e3
            nbytes = workloads.w4a16_bytes(m, n, k) - (m * n if fused else 0)  # fused: y is [M, N/2]
            flops = 2 * m * n * k
            ideal_us = max(nbytes / (peaks["hbm_gbs"] * 1e3), flops / (peaks["tflops"] * 1e6))
            rows.append({"linear": name, "n": n, "k": k, "m": m, "kernel": w4a16_kernel(m, n, k),
                         "us_per_call": round(us, 2), "gbs": round(nbytes / us / 1e3, 1),
                         "tflops": round(flops / us / 1e6, 1), "frac_of_roofline": round(ideal_us / us, 3)})
        del ws
        torch.cuda.empty_cache()
    return rows


def norm_quant_timing(args, rank: int, device, timer) -> dict:
    """RMSNorm + per-token INT8 on [NQ_ROWS, NQ_D] bf16, rotating over NQ_COPIES inputs (larger than L2 together),
    programmatic dependent launch."""
    from bpt_b200.kernels.norm_quant import rms_norm_int8

    gq = torch.Generator(device=device).manual_seed(1000 + rank)
    xs = [(torch.randn(NQ_ROWS, NQ_D, generator=gq, device=device) * 3).to(torch.bfloat16) for _ in range(NQ_COPIES)]
    w = (torch.rand(NQ_D, generator=gq, device=device) + 0.5).to(torch.bfloat16)
    outs = [(torch.empty(NQ_ROWS, NQ_D, dtype=torch.int8, device=device), torch.empty(NQ_ROWS, device=device))
            for _ in range(NQ_COPIES)]

    def call(i: int):
        rms_norm_int8(xs[i % NQ_COPIES], w, 1e-6, out=outs[i % NQ_COPIES], pdl=True)

    for i in range(3):
        call(i)
    ms = timer(call, args.steps) / args.steps
    del xs, outs
    nbytes = norm_quant_bytes(NQ_ROWS, NQ_D, False)
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"shape": f"[{NQ_ROWS}, {NQ_D}] bf16 -> int8 + fp32 scale per row", "us_per_call": round(ms * 1e3, 2),
            "gbs": round(gbs, 1), "frac_of_peak": round(gbs / measured_peaks()["hbm_gbs"], 3), "bytes": nbytes}


def column_parallel_timing(args, world: int, device, timer) -> dict:
    """The column-parallel W4A16 linear at the config-1 shape (6144 x 2048, M = 1): each rank holds 6144 / N rows,
    runs the streaming GEMV on them and NCCL all-gathers the [1, 6144 / N] blocks. Per-call device time (the slowest
    rank's, via the Timer's barrier), beside the local GEMV alone; every rank runs the same calls in the same order."""
    from bpt_b200.column_parallel import ColumnParallelW4A16Linear
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_linear

    g = torch.Generator(device=device).manual_seed(7)  # the same weight on every rank: each keeps its own rows
    copies = GEMV_COPIES
    layers = [ColumnParallelW4A16Linear(*quantize_w4a16(torch.randn(6144, 2048, generator=g, device=device) * 0.02),
                                        128) for _ in range(copies)]
    x = torch.randn(1, 2048, generator=g, device=device).to(torch.bfloat16)
    y = torch.empty(1, 6144, dtype=torch.bfloat16, device=device)
    part = torch.empty(1, 6144 // world, dtype=torch.bfloat16, device=device)

    def full(i):
        layers[i % copies](x, out=y, local_out=part)

    def local(i):
        lay = layers[i % copies]
        w4a16_linear(x, lay.qweight, lay.scales, lay.qzeros, out=part, pdl=True)

    for i in range(3):
        full(i)
        local(i)
    full_ms = timer(full, args.steps) / args.steps
    local_ms = timer(local, args.steps) / args.steps
    t = torch.tensor([full_ms, local_ms], device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    del layers
    return {"us_per_call": round(float(t[0]) * 1e3, 2), "local_gemv_us": round(float(t[1]) * 1e3, 2),
            "rows_per_rank": 6144 // world, "gather_bytes": 6144 * 2,
            "note": "M = 1: the all-gather of 12 KB is latency-bound and costs more than the weight bytes a rank saves"}


def decode_step_timing(args, rank: int, device: torch.device, timer) -> dict:
    """Config 5 on this rank: its own batch of 64 sequences (lengths shared by the ranks, weights and pool seeded by the
    rank), one graph-captured step per launch; device time of `decode_steps` steps with the GPU leading as for the
    other regions."""
    from bpt_b200.decode import Qwen3Decoder, Qwen3Dims

    g = torch.Generator().manual_seed(1000)  # the same lengths on every rank (weak scaling), weights and pool by rank
    lengths = torch.randint(1024, 8193, (64,), generator=g)
    dec = Qwen3Decoder(Qwen3Dims(), lengths, device=device, seed=rank, capacity=args.decode_steps + 8)
    dec.capture()
    for _ in range(3):
        dec.step()
    timer.barrier()
    kv0 = dec.kv_bytes_per_step()
    ms = timer(lambda i: dec.step(), args.decode_steps, host_s=1e-4)
    d = dec.dims
    grow = d.layers * dec.batch * 2 * d.kv_heads * d.head_dim  # one more token per sequence each step
    per_step = kv0 + (args.decode_steps - 1) * grow // 2 + dec.weight_bytes_per_step()  # mean KV read + weights
    dec.graph = None
    del dec
    torch.cuda.empty_cache()
    return {"decode_ms": ms, "decode_tokens": 64 * args.decode_steps, "decode_bytes": per_step * args.decode_steps}


# ---- the CPU baseline: the reference path restated (oracle port) on the host cores ------------------------------


def cpu_inputs(seed: int = 0):
    """The config-1 GEMV and the whole config-2 batch (32 sequences, lengths U[512, 4096]) on the CPU, with a pool
    holding exactly their pages."""
    from oracle import kv_formats as okv
    from oracle import w4a16 as ow4

    g = torch.Generator().manual_seed(seed)
    w = torch.randn(6144, 2048, generator=g) * 0.02
    qweight, scales, qzeros = ow4.pack_w4a16(*ow4.quantize_w4a16(w, 128))
    x = torch.randn(1, 2048, generator=g).to(torch.bfloat16)
    lengths = torch.randint(512, 4097, (32,), generator=g)
    need = ((lengths + 15) // 16).tolist()
    pages = sum(need)
    perm = torch.randperm(pages, generator=g)
    bt = torch.zeros(32, max(need), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(need):
        bt[i, :n] = perm[pos: pos + n].to(torch.int32)
        pos += n
    kpool = okv.fp8_store(torch.randn(pages, 16, 8, 128, generator=g), 1 / 64)
    vpool = okv.fp8_store(torch.randn(pages, 16, 8, 128, generator=g), 1 / 64)
    kv = okv.PagedKV("fp8", kpool, vpool, 1 / 64, 1 / 64, bt, 16)
    q = torch.randn(32, 16, 128, generator=g).to(torch.bfloat16)
    return (x, qweight, scales, qzeros), (q, kv, lengths)


def cpu_baseline(repeats: int = 3, inputs=None) -> dict:
    """The reference's plain-PyTorch path on the host cores (the oracle port): W4A16 dequantize + fp32 linear at the
    config-1 shape, and gather, dequantize, attend for the whole config-2 batch (same_config: the GPU step's shapes
    and distributions). Achieved GB/s over the same algorithmic bytes as the GPU metric, median of `repeats`."""
    from oracle import attention as oatt
    from oracle import w4a16 as ow4
    from bpt_b200.workloads import paged_bytes, w4a16_bytes

    torch.set_num_threads(os.cpu_count() or 1)
    (x, qweight, scales, qzeros), (q, kv, lengths) = inputs or cpu_inputs()
    nbytes = w4a16_bytes(1, 6144, 2048) + paged_bytes(lengths, 16, 8, 128, "fp8")
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        ow4.w4a16_linear(x, qweight, scales, qzeros, 128)
        oatt.paged_attend(q, kv, lengths, 1 / math.sqrt(128))
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {
        "value": round(nbytes / t / 1e9, 3),
        "unit": "GB/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "same_config": True,
        "sample": f"one full step: the config-1 GEMV and config-2 attention over all 32 sequences "
                  f"({int(lengths.sum())} tokens); median of {repeats}",
        "s_per_sample": round(t, 4),
    }


def norm_quant_cpu_baseline(repeats: int = 3) -> dict:
    """The reference's definition of rms_norm_int8 (kernels/reference.py:44-55, restated by the oracle) on the
    host cores, on the bench's [NQ_ROWS, NQ_D] bf16 shape: one full call, median of `repeats`."""
    from oracle import norm_quant as onq

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(1000)
    x = (torch.randn(NQ_ROWS, NQ_D, generator=g) * 3).to(torch.bfloat16)
    w = (torch.rand(NQ_D, generator=g) + 0.5).to(torch.bfloat16)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        onq.rms_norm_int8(x, w, 1e-6)
        times.append(time.perf_counter() - t0)
    s = statistics.median(times)
    return {"us_per_call": round(s * 1e6, 1), "gbs": round(norm_quant_bytes(NQ_ROWS, NQ_D, False) / s / 1e9, 2),
            "cores": torch.get_num_threads(), "kind": "port", "sample": "one full call, median of 3"}


def run_reference(args, rank: int, world: int) -> dict | None:
    """The reference arm: rank 0 alone times the CPU path on the host's cores (every step one full sample of the
    workload); the other ranks exit without work."""
    if rank != 0:
        return None
    inputs = cpu_inputs()
    for _ in range(max(args.warmup, 1)):
        cpu_baseline(repeats=1, inputs=inputs)
    samples = [cpu_baseline(repeats=1, inputs=inputs) for _ in range(args.steps)]
    value = statistics.median(s["value"] for s in samples)
    cores = samples[0]["cores"]
    return {
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(statistics.median(s["s_per_sample"] for s in samples) * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded)",
        "impl": "reference",
        "config": {"workload": WORKLOAD, "sample": samples[0]["sample"]},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "same_config": True,
                         "sample": samples[0]["sample"]},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---- single-kernel cases (for ncu) and sweep tables -----------------------------------------------------------------


def _case_time(fn, launches: int) -> float:
    """Mean device time per launch (us) of `launches` calls after one warm-up call (not a benchmark number)."""
    fn(0)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(launches):
        fn(i + 1)
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) * 1e3 / launches


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


def run_case(args) -> None:
    """One kernel on one workload, `--launches` times back to back (for ncu: -k on the kernel, -c on the launches),
    or a sweep that prints a markdown table (graph replay over rotating inputs larger than L2, PDL)."""
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_attention import attend, attend_workspace
    from bpt_b200.kernels.kv_write import empty_quant_kv, quantize_kv, quantize_kv_into, quantize_kv_paged
    from bpt_b200.kernels.norm_quant import rms_norm_int8
    from bpt_b200.kernels.w4a16 import quantize_w4a16, w4a16_gate_up_silu, w4a16_linear

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    peak = measured_peaks()["hbm_gbs"]
    name = args.case
    if name in ("attention-config2", "attention-config3"):
        # config 2: the bench's own three batches (rank 0's seeds), launch i on batch i mod 3, so a capture of three
        # launches averages exactly the batches the bench times; config 3: its first batch
        cases = ([workloads.config2(device=dev, seed=i) for i in range(ATTN_BATCHES)] if name.endswith("2")
                 else [workloads.config3(device=dev, seed=50)])
        b, hq, d = cases[0].q.shape
        tok = 4096 if name.endswith("2") else 32768
        out = torch.empty(b, hq, d, dtype=torch.bfloat16, device=dev)
        ws = attend_workspace(b, hq, d, -(-tok // 64), dev)
        us = _case_time(lambda i: attend(cases[i % len(cases)].q, cases[i % len(cases)].kv, cases[i % len(cases)].lengths,
                                         1.0 / math.sqrt(d), out=out, workspace=ws, tokens=tok), args.launches)
        print(f"{name}: {us:.1f} us per launch; algorithmic bytes per batch: {[c.bytes for c in cases]}")
    elif name == "gemv-config1":
        case = workloads.config1(device=dev)
        y = torch.empty(1, 6144, dtype=torch.bfloat16, device=dev)
        us = _case_time(lambda i: w4a16_linear(case.x, case.qweight, case.scales, case.qzeros, out=y), args.launches)
        print(f"{name}: {us:.2f} us per launch")
    elif name == "gemv-kernels":
        # config 1 as the bench's chain (40 rotating weight copies, each call waiting on its predecessor under PDL)
        # on the streaming tensor-core GEMV and on the CUDA-core kernel (packed fp32x2 FMAs over magic-number
        # unpacked codes), which the public API takes when the scales and zero points are not 16-byte aligned
        timer = Timer(dev, None)
        weights, x, _ = build_inputs(dev, seed=0, attention=False)
        y = torch.empty(1, 6144, dtype=torch.bfloat16, device=dev)

        def unaligned(t):
            buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=dev)
            view = buf[1:].view_as(t)
            view.copy_(t)
            return view

        variants = {"stream (aligned)": weights,
                    "CUDA cores (unaligned scales)": [(qw, unaligned(sc), unaligned(qz)) for qw, sc, qz in weights]}
        nbytes = workloads.w4a16_bytes(1, 6144, 2048)
        print("| kernel | us per chained call | GB/s | of HBM peak |\n|---|---|---|---|")
        for label, ws in variants.items():
            assert (ws[0][1].data_ptr() % 16 == 0) == label.startswith("stream"), label

            def call(i, ws=ws):
                qw, sc, qz = ws[i % GEMV_COPIES]
                w4a16_linear(x, qw, sc, qz, out=y, pdl=True)

            for i in range(5):
                call(i)
            us = timer(call, 200) * 1e3 / 200
            gbs = nbytes / us / 1e3
            print(f"| {label} | {us:.2f} | {gbs:.0f} | {gbs / peak:.1%} |", flush=True)
    elif name == "decode-step":
        # config 5 as the bench runs it (rank 0's batch): 3 warm-up steps after the capture, then `--launches` graph
        # replays (a launch list of these gives each kernel's share of the step)
        from bpt_b200.decode import Qwen3Decoder, Qwen3Dims

        g = torch.Generator().manual_seed(1000)
        lengths = torch.randint(1024, 8193, (64,), generator=g)
        dec = Qwen3Decoder(Qwen3Dims(), lengths, device=dev, seed=0, capacity=args.launches + 8)
        dec.capture()
        for _ in range(3):
            dec.step()
        torch.cuda.synchronize()
        us = _case_time(lambda i: dec.step(), args.launches)
        print(f"{name}: {us / 1e3:.3f} ms per step")
    elif name.startswith("gate-up-m"):
        m = int(name.split("-m")[1])
        g = torch.Generator(device=dev).manual_seed(0)
        qw = quantize_w4a16(torch.randn(12288, 2048, generator=g, device=dev) * 0.02, 128)
        x = torch.randn(m, 2048, generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty(m, 6144, dtype=torch.bfloat16, device=dev)
        us = _case_time(lambda i: w4a16_gate_up_silu(x, *qw, out=y), args.launches)
        print(f"{name}: {us:.2f} us per launch")
    elif name == "norm-quant":
        g = torch.Generator(device=dev).manual_seed(0)
        x = (torch.randn(NQ_ROWS, NQ_D, generator=g, device=dev) * 3).to(torch.bfloat16)
        w = (torch.rand(NQ_D, generator=g, device=dev) + 0.5).to(torch.bfloat16)
        out = (torch.empty(NQ_ROWS, NQ_D, dtype=torch.int8, device=dev), torch.empty(NQ_ROWS, device=dev))
        us = _case_time(lambda i: rms_norm_int8(x, w, 1e-6, out=out), args.launches)
        print(f"{name}: {us:.1f} us per launch")
    elif name == "kivi-sweep":
        print("| batch x tokens | bits | us per call | GB/s | of HBM peak |\n|---|---|---|---|---|")
        hq, hkv, d, t = 16, 8, 128, 32768
        for batch in (1, 8):
            for bits in (4, 8, 16):
                nbytes = kivi_bytes(batch, hkv, t, d, bits)
                copies = max(2, min(8, int(400e6 // nbytes)))
                g = torch.Generator(device=dev).manual_seed(batch * 100 + bits)
                caches = []
                for _ in range(copies):
                    k = torch.randn(batch, hkv, t, d, generator=g, device=dev).to(torch.bfloat16)
                    v = torch.randn(batch, hkv, t, d, generator=g, device=dev).to(torch.bfloat16)
                    caches.append(quantize_kv(k, v, bits))
                    del k, v
                q = torch.randn(batch, hq, d, generator=g, device=dev).to(torch.bfloat16)
                lengths = torch.full((batch,), t, dtype=torch.int32, device=dev)
                out = torch.empty(batch, hq, d, device=dev)

                def calls():
                    for kv in caches:
                        attend(q, kv, lengths, 1.0 / math.sqrt(d), out=out, tokens=t)

                us = _graph_us(calls, copies)
                gbs = nbytes / us / 1e3
                print(f"| {batch} x {t} | {bits} | {us:.2f} | {gbs:.0f} | {gbs / peak:.1%} |", flush=True)
                del caches
                torch.cuda.empty_cache()
    elif name == "kv-write-bulk":
        # the bulk paged FP8 write of the sweep (32 x 8 x 512 x 128 bf16 K and V), one input: a case for ncu
        hkv, d, bs, batch, q = 8, 128, 16, 32, 512
        g = torch.Generator(device=dev).manual_seed(1)
        kv = workloads.empty_pool("fp8", batch * q // bs + batch, bs, hkv, d, dev, None)
        k = torch.randn(batch, hkv, q, d, generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn(batch, hkv, q, d, generator=g, device=dev).to(torch.bfloat16)
        slot = torch.arange(batch * q, device=dev, dtype=torch.int32).view(batch, q)
        wb, wo = (slot // bs).contiguous(), (slot % bs).contiguous()
        us = _case_time(lambda i: quantize_kv_paged(k, v, kv, wb, wo), args.launches)
        print(f"{name}: {us:.1f} us per launch")
    elif name == "kv-write-sweep":
        print("| write | shape (B x Hkv x tokens x D, bf16 in) | us per call | GB/s | of HBM peak |\n|---|---|---|---|---|")
        hkv, d, bs = 8, 128, 16
        for kind in ("fp8", "int8"):
            for batch, q in ((64, 1), (32, 512)):
                elems = batch * hkv * q * d
                nbytes = 2 * elems * 2 + 2 * elems + (2 * batch * hkv * q * 2 if kind == "int8" else 0) + 2 * batch * q * 4
                copies = max(2, min(40, int(300e6 // nbytes)))
                g = torch.Generator(device=dev).manual_seed(batch + q)
                blocks = batch * q // bs + batch
                kvs = [workloads.empty_pool(kind, blocks, bs, hkv, d, dev, None) for _ in range(copies)]
                ks = [torch.randn(batch, hkv, q, d, generator=g, device=dev).to(torch.bfloat16) for _ in range(copies)]
                vs = [torch.randn(batch, hkv, q, d, generator=g, device=dev).to(torch.bfloat16) for _ in range(copies)]
                slot = torch.arange(batch * q, device=dev, dtype=torch.int32).view(batch, q)
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
            nbytes = 2 * batch * hkv * t * d * 2 + kivi_bytes(batch, hkv, t, d, bits)
            g = torch.Generator(device=dev).manual_seed(bits)
            ks = [torch.randn(batch, hkv, t, d, generator=g, device=dev).to(torch.bfloat16) for _ in range(2)]
            vs = [torch.randn(batch, hkv, t, d, generator=g, device=dev).to(torch.bfloat16) for _ in range(2)]
            caches = [empty_quant_kv(batch, hkv, t, d, bits, 32, dev) for _ in range(2)]

            def calls():
                for i in range(2):
                    quantize_kv_into(ks[i], vs[i], caches[i], 0)

            us = _graph_us(calls, 2)
            gbs = nbytes / us / 1e3
            print(f"| KIVI {bits}-bit quantize | {batch} x {hkv} x {t} x {d} | {us:.2f} | {gbs:.0f} | {gbs / peak:.1%} |",
                  flush=True)
            del ks, vs, caches
            torch.cuda.empty_cache()
    elif name == "norm-quant-sweep":
        print("| rows x d (bf16) | residual | us per call | GB/s | of HBM peak |\n|---|---|---|---|---|")
        for rows, d, residual in [(64, 2048, False), (64, 2048, True), (256, 2048, False), (4096, 2048, False),
                                  (16384, 2048, False), (16384, 2048, True), (16384, 6144, False)]:
            nbytes = norm_quant_bytes(rows, d, residual)
            copies = max(2, min(40, int(300e6 // nbytes)))
            g = torch.Generator(device=dev).manual_seed(rows + d)
            xs = [(torch.randn(rows, d, generator=g, device=dev) * 3).to(torch.bfloat16) for _ in range(copies)]
            ds = [torch.randn(rows, d, generator=g, device=dev).to(torch.bfloat16) for _ in range(copies)]
            w = (torch.rand(d, generator=g, device=dev) + 0.5).to(torch.bfloat16)
            outs = [(torch.empty(rows, d, dtype=torch.int8, device=dev), torch.empty(rows, device=dev))
                    for _ in range(copies)]
            sums = [torch.empty_like(xs[0]) for _ in range(copies)]

            def calls():
                for i in range(copies):
                    if residual:
                        rms_norm_int8(xs[i], w, 1e-6, out=outs[i], delta=ds[i], x_out=sums[i], pdl=True)
                    else:
                        rms_norm_int8(xs[i], w, 1e-6, out=outs[i], pdl=True)

            us = _graph_us(calls, copies)
            gbs = nbytes / us / 1e3
            print(f"| {rows} x {d} | {'yes' if residual else 'no'} | {us:.2f} | {gbs:.0f} | {gbs / peak:.1%} |",
                  flush=True)
            del xs, ds, outs, sums
            torch.cuda.empty_cache()
    else:
        raise SystemExit(f"unknown case {name!r}")


CASES = ["attention-config2", "attention-config3", "gemv-config1", "gemv-kernels", "decode-step", "gate-up-m16", "gate-up-m64", "gate-up-m256",
         "norm-quant", "kivi-sweep", "kv-write-bulk", "kv-write-sweep", "norm-quant-sweep"]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--decode-steps", type=int, default=20, help="config-5 decode steps timed (0: skip)")
    ap.add_argument("--quick", action="store_true", help="leave out the config-3, config-4 and rms_norm_int8 regions")
    ap.add_argument("--case", choices=CASES, help="run one kernel case or sweep instead of the benchmark")
    ap.add_argument("--launches", type=int, default=4, help="launches of a --case kernel")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.no_decode = args.decode_steps <= 0
    if args.case:
        run_case(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}; using WORLD_SIZE", file=sys.stderr)

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    from datetime import timedelta

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    try:
        line = run_ours(args, rank, world, device)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
