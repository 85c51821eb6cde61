"""Benchmark of fastserve's decode hot path on B200: W4A16 GEMV (config 1) + paged FP8-KV decode attention
(config 2), one step = one GEMV and one attention over one batch, inputs resident in HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU; weak scaling, no collective)

Prints one JSON line (rank 0). `value` is whole-job achieved HBM bandwidth: the algorithmic bytes of every
rank's steps over the slowest rank's device time. `e2e` is the same metric through the public Python API with
this step's inputs copied from pinned host memory and the results copied back inside the timed region (one
staging copy each way: the kernels read and write views of one device buffer per direction).
`--impl reference` times the reference's CPU path (the oracle port: dequantize-then-matmul and gather,
dequantize, attend) on the host cores, on a bounded sample of the same workload.

Inputs larger than L2: the GEMV rotates over 40 weight copies (262 MB) and the attention over 3 batches with
their own pools (about 450 MB of KV touched per cycle), so no step finds its data in the 126 MB L2.

`kernels.rms_norm_int8` times the next row past the path in its own region (RMSNorm + per-token INT8 of
[16384, 2048] bf16 rows, three rotating inputs of 64 MB), with the reference's CPU definition beside it at N=1.
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
NQ_ROWS, NQ_D, NQ_COPIES = 16384, 2048, 3  # rms_norm_int8: 3 x 64 MB of bf16 rows rotate (above L2)


def norm_quant_bytes(rows: int, d: int, residual: bool) -> int:
    """rms_norm_int8's algorithmic bytes: bf16 x read, int8 codes and fp32 scales written, the weight once."""
    return rows * d * 3 + rows * 4 + d * 2 + (4 * rows * d if residual else 0)
PROFILE_SUMMARY = ROOT / "profiles" / "paged_attention_fp8_config2.md"


def measured_peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic() -> int | None:
    """DRAM bytes per launch of the attention kernel from the committed ncu summary (a line
    `traffic_bytes_per_launch: N`), scaled to this run's workload by the caller."""
    if not PROFILE_SUMMARY.exists():
        return None
    for line in PROFILE_SUMMARY.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            return int(line.split(":", 1)[1].strip().replace(",", ""))
    return None


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


# ---- our arm ------------------------------------------------------------------------------------------------------


def build_inputs(device: torch.device, seed: int):
    from bpt_b200 import workloads
    from bpt_b200.kernels.w4a16 import quantize_w4a16

    g = torch.Generator(device=device).manual_seed(seed)
    weights = []
    for _ in range(GEMV_COPIES):
        w = torch.randn(6144, 2048, generator=g, device=device) * 0.02
        weights.append(quantize_w4a16(w, 128))
    x = torch.randn(1, 2048, generator=g, device=device).to(torch.bfloat16)
    attn = [workloads.config2(device=device, seed=seed * 100 + i) for i in range(ATTN_BATCHES)]
    return weights, x, attn


def run_ours(args, rank: int, world: int, device: torch.device) -> dict | None:
    from bpt_b200 import workloads
    from bpt_b200.kernels.kv_attention import attend, attend_workspace, paged_split
    from bpt_b200.kernels.w4a16 import w4a16_linear

    dist = torch.distributed if world > 1 else None
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

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)

    for i in range(max(args.warmup, 3)):
        step(i)
    barrier()
    # host time to enqueue one step, so each timed region can start with the GPU far enough behind the host that
    # its launches run back to back on the device (the events then time kernels, not Python launch overhead)
    t0 = time.perf_counter()
    for i in range(8):
        step(i)
    host_step_s = (time.perf_counter() - t0) / 8
    barrier()
    clock_khz = torch.cuda.get_device_properties(device).clock_rate or 2_000_000
    lead_cycles = int(min(0.5, 2.0 * host_step_s * args.steps + 1e-3) * clock_khz * 1e3)
    stream = torch.cuda.current_stream(device)

    def timed(fn) -> float:
        """Device time of K launches of fn (ms): events on the launching stream around the whole sequence."""
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(lead_cycles)  # the GPU idles (outside the region) while the host enqueues the launches
        start.record(stream)
        for k in range(args.steps):
            fn(k)
        end.record(stream)
        barrier()
        return start.elapsed_time(end)

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
        total_ms = timed(step)
        attn_total_ms = timed(attention)
        gemv_total_ms = timed(gemv)
    gemv_ms = [gemv_total_ms / args.steps]
    attn_ms = [attn_total_ms / args.steps]

    # the next row past the path: RMSNorm + per-token INT8 on [NQ_ROWS, NQ_D] bf16, rotating over NQ_COPIES inputs
    # (larger than L2 together), programmatic dependent launch
    from bpt_b200.kernels.norm_quant import rms_norm_int8

    gq = torch.Generator(device=device).manual_seed(1000 + rank)
    nq_x = [(torch.randn(NQ_ROWS, NQ_D, generator=gq, device=device) * 3).to(torch.bfloat16) for _ in range(NQ_COPIES)]
    nq_w = (torch.rand(NQ_D, generator=gq, device=device) + 0.5).to(torch.bfloat16)
    nq_out = [(torch.empty(NQ_ROWS, NQ_D, dtype=torch.int8, device=device), torch.empty(NQ_ROWS, device=device))
              for _ in range(NQ_COPIES)]

    def norm_quant(i: int):
        rms_norm_int8(nq_x[i % NQ_COPIES], nq_w, 1e-6, out=nq_out[i % NQ_COPIES], pdl=True)

    for i in range(3):
        norm_quant(i)
    nq_ms = [timed(norm_quant) / args.steps]
    del nq_x, nq_out
    my_bytes = sum(gemv_bytes + attn_bytes[k % ATTN_BATCHES] for k in range(args.steps))

    # end to end: the public API with host buffers, the step's inputs H2D and results D2H inside the region. As a
    # serving loop stages them, a step's inputs (x, q, lengths, block table) sit in one pinned buffer and cross in
    # one copy into one device buffer that the kernels read through views; the two results (y, out) are views of
    # one device buffer and come back in one copy.
    def layout(parts):  # [(name, bytes)] -> ({name: offset}, total), each part 256-byte aligned
        offs, at = {}, 0
        for name, nb in parts:
            offs[name] = at
            at += (nb + 255) // 256 * 256
        return offs, at

    def view(buf, off, like):
        return buf[off: off + like.numel() * like.element_size()].view(like.dtype).view(like.shape)

    stage_in, pin_in, e2e_cases = [], [], []
    for c in attn:  # each batch its own layout (block-table widths differ)
        ioff, in_total = layout([("x", x.numel() * 2), ("q", c.q.numel() * 2), ("lengths", c.lengths.numel() * 4),
                                 ("table", c.kv.block_table.numel() * 4)])
        dev = torch.empty(in_total, dtype=torch.uint8, device=device)
        xv, qv, lv, tv = (view(dev, ioff["x"], x), view(dev, ioff["q"], c.q), view(dev, ioff["lengths"], c.lengths),
                          view(dev, ioff["table"], c.kv.block_table))
        xv.copy_(x), qv.copy_(c.q), lv.copy_(c.lengths), tv.copy_(c.kv.block_table)
        stage_in.append(dev)
        pin_in.append(dev.cpu().pin_memory())
        e2e_cases.append((xv, qv, lv, dataclasses.replace(c.kv, block_table=tv)))
    ooff, out_total = layout([("y", y.numel() * 2), ("out", out.numel() * 2)])
    stage_out = torch.empty(out_total, dtype=torch.uint8, device=device)
    y_v, out_v = view(stage_out, ooff["y"], y), view(stage_out, ooff["out"], out)
    pin_out = torch.empty(out_total, dtype=torch.uint8).pin_memory()
    # the bytes that cross per step (padding included), averaged over the rotating batches
    h2d, d2h = round(sum(t.numel() for t in stage_in) / len(stage_in)), out_total

    def e2e_step(i: int):
        j = i % ATTN_BATCHES
        xv, qv, lv, kv = e2e_cases[j]
        qw, sc, qz = weights[i % GEMV_COPIES]
        stage_in[j].copy_(pin_in[j], non_blocking=True)
        w4a16_linear(xv, qw, sc, qz, out=y_v, pdl=True)
        attend(qv, kv, lv, scale, out=out_v, tokens=4096, split=split, pdl=True, kv_ready=True)
        pin_out.copy_(stage_out, non_blocking=True)

    for i in range(3):
        e2e_step(i)
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for k in range(args.steps):
        e2e_step(k)
    e_end.record(stream)
    barrier()
    e2e_ms = e_start.elapsed_time(e_end)

    local = {
        "total_ms": total_ms,
        "e2e_ms": e2e_ms,
        "bytes": my_bytes,
        "gemv_ms": gemv_ms,
        "attn_ms": attn_ms,
        "nq_ms": nq_ms,
        "clocks": sampler.summary(),
    }
    del weights, attn, stage_in, pin_in, e2e_cases, stage_out, pin_out
    torch.cuda.empty_cache()
    if not args.no_decode:
        local.update(decode_step_timing(args, rank, device, barrier))
    gathered = gather_ranks(local, dist)
    if rank != 0:
        return None

    whole = combine_ranks(gathered)
    t_max, e_max, all_bytes = whole["total_ms"], whole["e2e_ms"], whole["bytes"]
    gbs = all_bytes / (t_max * 1e-3) / 1e9
    e2e_gbs = all_bytes / (e_max * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()
    attn_avg_ms = statistics.fmean(gathered[0]["attn_ms"])
    gemv_avg_ms = statistics.fmean(gathered[0]["gemv_ms"])
    nq_avg_ms = statistics.fmean(gathered[0]["nq_ms"])
    nq_bytes = norm_quant_bytes(NQ_ROWS, NQ_D, False)
    attn_bytes_avg = statistics.fmean(attn_bytes)
    achieved = attn_bytes_avg / (attn_avg_ms * 1e-3) / 1e9
    traffic = profiled_traffic()
    clocks = gathered[0]["clocks"]
    reasons = sorted({r for g in gathered for r in g["clocks"]["reasons"]})
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
        "kernels": {
            "w4a16_gemv": {"us_per_call": round(gemv_avg_ms * 1e3, 2),
                           "gbs": round(gemv_bytes / (gemv_avg_ms * 1e-3) / 1e9, 1),
                           "frac_of_peak": round(gemv_bytes / (gemv_avg_ms * 1e-3) / 1e9 / peak, 3),
                           "bytes": gemv_bytes},
            "paged_attention_fp8": {"us_per_call": round(attn_avg_ms * 1e3, 2), "gbs": round(achieved, 1),
                                    "frac_of_peak": round(achieved / peak, 3), "bytes": round(attn_bytes_avg)},
            "rms_norm_int8": {"shape": f"[{NQ_ROWS}, {NQ_D}] bf16 -> int8 + fp32 scale per row",
                              "us_per_call": round(nq_avg_ms * 1e3, 2),
                              "gbs": round(nq_bytes / (nq_avg_ms * 1e-3) / 1e9, 1),
                              "frac_of_peak": round(nq_bytes / (nq_avg_ms * 1e-3) / 1e9 / peak, 3), "bytes": nq_bytes},
        },
        "roofline": {
            "kernel": "paged_attn_persistent_kernel<128, 2, FP8> (fused split merge)",
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind,
            "unit": "GB/s",
            "frac": round(achieved / peak, 3),
            "traffic": None if traffic is None else traffic,
        },
        "e2e": {"value": round(e2e_gbs, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e_max / args.steps, 5)},
        "gpu_launches": 2 * args.steps,
        "gpu_launches_note": "the step region; the per-kernel regions launch K more of each kernel",
        "clocks": {"sm_mhz": clocks["sm_mhz"], "sm_max_mhz": clocks["sm_max_mhz"], "reasons": reasons,
                   "samples": clocks["samples"], "window": "0.3 s soak of the same step + the timed region"},
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
            "bytes_per_step_per_gpu": gathered[0]["decode_bytes"] // args.decode_steps,
            "steps": args.decode_steps,
            "scaling": "weak",
        }
    if world == 1:
        line["cpu_baseline"] = cpu_baseline(sample_seqs=4)
        line["kernels"]["rms_norm_int8"]["cpu_baseline"] = norm_quant_cpu_baseline()
    return line


def decode_step_timing(args, rank: int, device: torch.device, barrier) -> dict:
    """Config 5 on this rank: its own batch of 64 sequences (seeded by the rank), one graph-captured step per
    launch; device time of `decode_steps` steps with the GPU leading as for the other regions."""
    from bpt_b200.decode import Qwen3Decoder, Qwen3Dims

    g = torch.Generator().manual_seed(1000 + rank)
    lengths = torch.randint(1024, 8193, (64,), generator=g)
    dec = Qwen3Decoder(Qwen3Dims(), lengths, device=device, seed=rank, capacity=args.decode_steps + 8)
    dec.capture()
    for _ in range(3):
        dec.step()
    barrier()
    kv0 = dec.kv_bytes_per_step()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(int(2e6))
    start.record()
    for _ in range(args.decode_steps):
        dec.step()
    end.record()
    barrier()
    ms = start.elapsed_time(end)
    d = dec.dims
    grow = d.layers * dec.batch * 2 * d.kv_heads * d.head_dim  # one more token per sequence each step
    per_step = kv0 + (args.decode_steps - 1) * grow // 2 + dec.weight_bytes_per_step()  # mean KV read + weights
    dec.graph = None
    del dec
    torch.cuda.empty_cache()
    return {"decode_ms": ms, "decode_tokens": 64 * args.decode_steps, "decode_bytes": per_step * args.decode_steps}


# ---- the CPU baseline: the reference path restated (oracle port) on the host cores ------------------------------


def cpu_baseline(sample_seqs: int = 4, repeats: int = 3) -> dict:
    """The reference's plain-PyTorch path on the host cores (the oracle port): W4A16 dequantize + fp32 linear at
    the config-1 shape, and gather, dequantize, attend, merge for `sample_seqs` sequences of a config-2 batch.
    Returns achieved GB/s over the same algorithmic bytes as the GPU metric."""
    from oracle import attention as oatt
    from oracle import kv_formats as okv
    from oracle import w4a16 as ow4

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    w = torch.randn(6144, 2048, generator=g) * 0.02
    codes, scales, zeros = ow4.quantize_w4a16(w, 128)
    qweight, scales, qzeros = ow4.pack_w4a16(codes, scales, zeros)
    x = torch.randn(1, 2048, generator=g).to(torch.bfloat16)
    # a config-2 batch restricted to `sample_seqs` sequences, pool holding exactly their pages
    lengths = torch.randint(512, 4097, (32,), generator=g)[:sample_seqs]
    pages = int(((lengths + 15) // 16).sum())
    table = torch.randperm(pages, generator=g)
    width = int((lengths.max() + 15) // 16)
    bt = torch.zeros(sample_seqs, width, dtype=torch.int32)
    pos = 0
    for i, n in enumerate(((lengths + 15) // 16).tolist()):
        bt[i, :n] = table[pos : pos + n].to(torch.int32)
        pos += n
    kpool = okv.fp8_store(torch.randn(pages, 16, 8, 128, generator=g), 1 / 64)
    vpool = okv.fp8_store(torch.randn(pages, 16, 8, 128, generator=g), 1 / 64)
    kv = okv.PagedKV("fp8", kpool, vpool, 1 / 64, 1 / 64, bt, 16)
    q = torch.randn(sample_seqs, 16, 128, generator=g).to(torch.bfloat16)
    from bpt_b200.workloads import paged_bytes, w4a16_bytes

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
        "sample": f"config-1 GEMV (full) + config-2 attention over {sample_seqs} of 32 sequences "
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
    if rank != 0:
        return None
    for _ in range(max(args.warmup, 1)):
        cpu_baseline(sample_seqs=4, repeats=1)
    samples = [cpu_baseline(sample_seqs=4, repeats=1) for _ in range(args.steps)]
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
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "sample": samples[0]["sample"]},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--decode-steps", type=int, default=20, help="config-5 decode steps timed (0: skip)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.no_decode = args.decode_steps <= 0

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
