#!/usr/bin/env python
"""Benchmark of the KernelForge hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

Headline: the RMSNorm bf16 sweep, rows x hidden in
{4096, 32768, 262144} x {1024, 2048, 4096, 8192}. One STEP normalises all 12 sweep tensors
once (18.4 GB of HBM traffic per GPU, far above the 126 MB L2). ``value`` is the aggregate
achieved HBM GB/s over all ranks with inputs resident in HBM; ``e2e`` is the same metric with
the inputs copied from pinned host memory and the outputs copied back inside the timed region.

Secondary workloads in the same line (``workloads``): SANA linear attention configs
(B=4,H=36,N=4096) and (B=2,H=70,N=16384), bf16 in/out, each step one ``qkv_attn_matmul`` call
(replayed from a CUDA graph); FlashAttention JVP (B=4,H=16,N=4096,D in {64,128}, bf16,
non-causal), each step one standalone ``flash_attention_jvp`` call (TFLOP/s over 5 GEMMs) or
one ``flash_attention_fwd_jvp`` call (6 GEMMs); FlashAttention backward on the same configs, each
step one ``_flash_attn_backward`` call (5 GEMMs); ``--flash-attn-comparator`` also times
flash_attn's own backward on the same tensors.

Multi-GPU: one process per GPU (torchrun), weak scaling -- every rank processes its own
full-size shard, no collective on the data path; NCCL only takes the max of the per-rank
device times and gathers per-rank output checksums after the timed region.

``--impl reference`` times the reference algorithm's CPU restatement (``oracle/``) on the
host cores on a bounded sample of the same workload (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
BASELINE_METRIC = "achieved HBM GB/s (RMSNorm, SANA-attn) & TFLOP/s (FA-JVP) vs B200 peak, 1–8 GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1024 * 1024

SWEEP_ROWS = (4096, 32768, 262144)
SWEEP_HIDDEN = (1024, 2048, 4096, 8192)
SANA_CONFIGS = (
    {"name": "sana_cfg1", "B": 4, "H": 36, "N": 4096, "D": 32},
    {"name": "sana_cfg2", "B": 2, "H": 70, "N": 16384, "D": 32},
    # One of the reference harness's own shapes (SANA test.py:184-186: batch 1, 2240 channels =
    # 70 heads, 4096 tokens): fewer heads than SMs, so the one-launch path runs in clusters.
    {"name": "sana_harness_b1h70", "B": 1, "H": 70, "N": 4096, "D": 32},
)

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from `ncu --set full`
# captures of the `--case ncu-small` shapes. RMSNorm: the 32768 x 8192 capture (536,926,976 read +
# 486,499,328 written) scaled by rows to the dominant 262144 x 8192 launch (x 8; every row is read
# once and written once, so traffic is linear in rows). SANA cfg1: the one-launch kernel of a call
# at the bench size itself (113,272,832 read + 7,127,808 written; most of the 37.7 MB output is
# still in L2 when the kernel ends).
RMSNORM_NCU_TRAFFIC_BYTES = 8 * (536_926_976 + 486_499_328)
SANA_NCU_TRAFFIC_BYTES = {"sana_cfg1": 113_272_832 + 7_127_808}
# RMSNorm backward at the bench size, from the capture in profiles/rmsnorm_bwd_vec_32768x8192_bf16.md.
RMSNORM_BWD_NCU_TRAFFIC_BYTES = 1_073_874_000 + 503_786_496


def sana_launches_per_call(B, H, N):
    """Kernel launches of one default-schedule qkv_attn_matmul call (bf16, head dim 32), as the
    library plans it on this device (kf_sana_linattn_plan)."""
    from kernelforge_b200.SANA_LinearAttention import QKVAttnMatmul

    return QKVAttnMatmul(B, H, 32, N, 1e-15, "bfloat16", "bfloat16").plan()[0]


# ---------------------------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------------------------
def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except (OSError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.enabled = self.world > 1

    def init(self):
        if self.enabled:
            torch.cuda.set_device(self.local_rank)
            torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=180),
                                                 device_id=torch.device("cuda", self.local_rank))
        else:
            torch.cuda.set_device(0)

    def barrier(self):
        if self.enabled:
            torch.distributed.barrier()

    def max(self, value: float) -> float:
        if not self.enabled:
            return value
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def gather(self, value: float):
        if not self.enabled:
            return [value]
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        out = [torch.zeros_like(t) for _ in range(self.world)]
        torch.distributed.all_gather(out, t)
        return [float(x.item()) for x in out]

    def close(self):
        if self.enabled:
            torch.distributed.destroy_process_group()


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the timed regions run."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [line.strip().split(", ") for line in self.file.read().splitlines() if line.strip()]
        os.unlink(self.file.name)
        samples = []
        for r in rows:
            try:
                samples.append(dict(sm=float(r[1]), smax=float(r[2]), util=float(r[4]),
                                    hw=r[6] == "Active", hwt=r[7] == "Active", swt=r[8] == "Active",
                                    pcap=r[9] == "Active"))
            except (IndexError, ValueError):
                continue
        if not samples:
            return None
        loaded = [s for s in samples if s["util"] >= 50] or samples
        reasons = sorted({name for s in loaded for name, key in (("hw_slowdown", "hw"),
                          ("hw_thermal_slowdown", "hwt"), ("sw_thermal_slowdown", "swt"),
                          ("sw_power_cap", "pcap")) if s[key]})
        return {"sm_mhz": statistics.median(s["sm"] for s in loaded),
                "sm_max_mhz": max(s["smax"] for s in loaded), "reasons": reasons,
                "samples": len(samples), "samples_under_load": len([s for s in samples if s["util"] >= 50])}


def time_region(step, steps, warmup, dist, dominant=None):
    """Warm up, then time exactly `steps` calls of step(i) between barriers + synchronize.

    Returns (max-over-ranks ms per step, average ms of the dominant launch or None)."""
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if dominant is not None:
        dominant.clear()
    start.record()
    for i in range(steps):
        step(i)
    end.record()
    end.synchronize()
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(start.elapsed_time(end)) / steps
    dom = None
    if dominant:
        dom = dist.max(sum(a.elapsed_time(b) for a, b in dominant) / len(dominant))
    return ms, dom


class LaunchTimer(list):
    """Collects (start, end) CUDA event pairs around the dominant kernel's launches."""

    def around(self, fn):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        out = fn()
        b.record()
        self.append((a, b))
        return out


def roofline(alg_bytes_or_flops, ms, peak, unit, bound, traffic=None):
    achieved = alg_bytes_or_flops / (ms / 1e3) / 1e9 if unit == "GB/s" else alg_bytes_or_flops / (ms / 1e3) / 1e12
    return {"bound": bound, "achieved": round(achieved, 1), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic}


def cpu_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


# ---------------------------------------------------------------------------------------------
# RMSNorm sweep
# ---------------------------------------------------------------------------------------------
# --case ncu-small: one small configuration per workload for `ncu --set full` captures (inputs
# still larger than L2, a few GB on the device at most). Not a benchmark line.
SMALL = {"rows": (32768,), "hidden": (8192,)}
CASE = "full"


def sweep_points():
    if CASE == "ncu-small":
        return [(r, h) for r in SMALL["rows"] for h in SMALL["hidden"]]
    return [(r, h) for r in SWEEP_ROWS for h in SWEEP_HIDDEN]


def rmsnorm_bytes(rows, hidden):
    return 2 * rows * hidden * 2 + 2 * hidden


def bench_rmsnorm(args, dist, peaks, peak_kind):
    from kernelforge_b200.rmsnorm import rms_norm, rmsnorm_into

    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(1234 + dist.rank)
    xs, ws, ys = [], [], []
    for rows, hidden in sweep_points():
        xs.append(torch.randn(rows, hidden, device=dev, dtype=torch.bfloat16, generator=gen))
        ws.append((1 + 0.1 * torch.randn(hidden, device=dev, generator=gen)).to(torch.bfloat16))
        ys.append(torch.empty(rows, hidden, device=dev, dtype=torch.bfloat16))
    dominant_index = len(xs) - 1  # the largest tensor (262144 x 8192 in the sweep)
    timer = LaunchTimer()

    def step(_):
        for j, (x, w, y) in enumerate(zip(xs, ws, ys)):
            if j == dominant_index:
                timer.around(lambda: rmsnorm_into(x, w, y, 1e-6))
            else:
                rmsnorm_into(x, w, y, 1e-6)

    ms, dom_ms = time_region(step, args.steps, args.warmup, dist, timer)
    per_gpu_bytes = sum(rmsnorm_bytes(r, h) for r, h in sweep_points())
    value = dist.world * per_gpu_bytes / (ms / 1e3) / 1e9
    checksums = dist.gather(float(sum(y.float().sum().item() for y in ys[:3])))
    dom_bytes = rmsnorm_bytes(*sweep_points()[dominant_index])
    result = {
        "value": round(value, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "gpu_launches": len(xs) * args.steps,
        "roofline": roofline(dom_bytes, dom_ms, peaks["hbm_gbs"], "GB/s", "hbm",
                             RMSNORM_NCU_TRAFFIC_BYTES),
        "roofline_note": f"dominant launch rmsnorm 262144x8192 bf16, {dom_ms * 1e3:.1f} us avg; "
                         f"peak = {peak_kind} HBM copy GB/s",
        "gathered_checksums": len(checksums),
    }
    if not args.no_e2e:
        result["e2e"] = rmsnorm_e2e(args, dist, xs, ws, rms_norm)
    del xs, ys
    torch.cuda.empty_cache()
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = rmsnorm_cpu_baseline(seconds=args.cpu_seconds)
    return result


def rmsnorm_e2e(args, dist, xs, ws, rms_norm):
    """Same sweep through the public API, inputs from pinned host memory, outputs back to host."""
    dev = xs[0].device
    biggest = max(x.numel() for x in xs)
    try:
        host_in = torch.empty(biggest, dtype=torch.bfloat16, pin_memory=True)
        host_out = torch.empty(biggest, dtype=torch.bfloat16, pin_memory=True)
    except RuntimeError as exc:
        return {"value": None, "unit": "GB/s", "error": f"pinned host allocation failed: {exc}"}
    host_in.copy_(xs[-1].view(-1))  # real input data in the pinned staging buffer
    dev_in = [torch.empty_like(x) for x in xs]
    kernels = [rms_norm(1, x.shape[0], x.shape[1], 1e-6, "bfloat16") for x in xs]
    h2d = sum(x.numel() * 2 for x in xs)
    d2h = h2d

    def step(_):
        for x_dev, w, kern in zip(dev_in, ws, kernels):
            n = x_dev.numel()
            x_dev.view(-1).copy_(host_in[:n], non_blocking=True)
            y = kern(x_dev.view(1, *x_dev.shape), w)
            host_out[:n].copy_(y.view(-1), non_blocking=True)

    steps = max(2, min(args.steps, args.e2e_steps))
    ms, _ = time_region(step, steps, min(args.warmup, 2), dist)
    per_gpu = sum(rmsnorm_bytes(r, h) for r, h in sweep_points())
    del dev_in
    return {"value": round(dist.world * per_gpu / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "ms_per_step": round(ms, 3), "api": "kernelforge_b200.rmsnorm.rms_norm(...)(X, Weight)"}


def rmsnorm_cpu_sample_rows():
    return 1024


def rmsnorm_cpu_baseline(seconds=10.0):
    """oracle.rmsnorm on the host cores over a bounded sample: the first 1024 rows of each sweep
    tensor (fp32 statistics, bf16 in/out), repeated until ~`seconds` elapsed."""
    from oracle.rmsnorm import rmsnorm_forward

    cores = cpu_threads()
    g = torch.Generator().manual_seed(0)
    rows = rmsnorm_cpu_sample_rows()
    data = [(torch.randn(min(rows, r), h, generator=g).to(torch.bfloat16),
             (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16)) for r, h in sweep_points()]
    nbytes = sum(rmsnorm_bytes(x.shape[0], x.shape[1]) for x, _ in data)
    for x, w in data:  # warm-up
        rmsnorm_forward(x, w, 1e-6)
    t0 = time.perf_counter()
    reps = 0
    while True:
        for x, w in data:
            rmsnorm_forward(x, w, 1e-6)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"first {rows} rows of each of the 12 sweep tensors (bf16), {reps} passes of "
                      f"{nbytes / 1e6:.0f} MB, oracle/rmsnorm.py (torch CPU, {cores} threads)"}


# RMSNorm backward (no counterpart in the reference): one BASELINE sweep shape, bf16.
RMSNORM_BWD_CONFIG = {"rows": 32768, "hidden": 8192}


def rmsnorm_bwd_bytes(rows, hidden):
    """x and dy read, dx written (bf16); the weight and dweight are negligible."""
    return 3 * rows * hidden * 2 + 2 * 2 * hidden


def bench_rmsnorm_bwd(args, dist, peaks, peak_kind):
    from kernelforge_b200.rmsnorm import rmsnorm_backward

    dev = torch.device("cuda", torch.cuda.current_device())
    rows, hidden = RMSNORM_BWD_CONFIG["rows"], RMSNORM_BWD_CONFIG["hidden"]
    gen = torch.Generator(device=dev).manual_seed(4321 + dist.rank)
    x = torch.randn(rows, hidden, device=dev, dtype=torch.bfloat16, generator=gen)
    dy = torch.randn(rows, hidden, device=dev, dtype=torch.bfloat16, generator=gen)
    w = (1 + 0.1 * torch.randn(hidden, device=dev, generator=gen)).to(torch.bfloat16)
    call = lambda: rmsnorm_backward(dy, x, w, 1e-6)  # noqa: E731
    timer = LaunchTimer()
    ms, dom_ms = time_region(lambda _: timer.around(call), args.steps, args.warmup, dist, timer)
    nbytes = rmsnorm_bwd_bytes(rows, hidden)
    result = {
        "value": round(dist.world * nbytes / (ms / 1e3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "gpu_launches": 2 * args.steps,
        "config": {"rows": rows, "hidden": hidden, "dtype": "bf16", "eps": 1e-6,
                   "call": "rmsnorm_backward(dy, x, weight) -> (dx, dweight)",
                   "bytes_per_step": nbytes, "l2": "inputs larger than L2 (x, dy 537 MB each)"},
        "roofline": roofline(nbytes, dom_ms, peaks["hbm_gbs"], "GB/s", "hbm", RMSNORM_BWD_NCU_TRAFFIC_BYTES),
        "roofline_note": f"x and dy read and dx written once per call; one call = 2 launches (dx with per-CTA "
                         f"dweight partials, then their fixed-order sum), {dom_ms * 1e3:.1f} us avg per call; "
                         f"peak = {peak_kind} HBM copy GB/s",
    }
    if not args.no_e2e:
        host_x, host_dy = x.cpu().pin_memory(), dy.cpu().pin_memory()
        host_dx = torch.empty_like(host_x).pin_memory()
        dev_x, dev_dy = torch.empty_like(x), torch.empty_like(dy)

        def e2e_step(_):
            dev_x.copy_(host_x, non_blocking=True)
            dev_dy.copy_(host_dy, non_blocking=True)
            dx, _ = rmsnorm_backward(dev_dy, dev_x, w, 1e-6)
            host_dx.copy_(dx, non_blocking=True)

        steps = max(3, min(args.steps, args.e2e_steps))
        ems, _ = time_region(e2e_step, steps, args.warmup, dist)
        result["e2e"] = {"value": round(dist.world * nbytes / (ems / 1e3) / 1e9, 2), "unit": "GB/s",
                         "h2d_bytes_per_step": 2 * x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2,
                         "steps": steps, "ms_per_step": round(ems, 3),
                         "api": "kernelforge_b200.rmsnorm.rmsnorm_backward"}
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = rmsnorm_bwd_cpu_baseline(seconds=args.cpu_seconds / 2)
    del x, dy
    torch.cuda.empty_cache()
    return result


def rmsnorm_bwd_cpu_baseline(seconds=5.0):
    """oracle.rmsnorm.rmsnorm_backward (float64 autograd) on the host cores: 256-row samples of the
    bench shape, repeated until ~`seconds` elapsed."""
    from oracle.rmsnorm import rmsnorm_backward

    cores = cpu_threads()
    g = torch.Generator().manual_seed(0)
    rows, hidden = 256, RMSNORM_BWD_CONFIG["hidden"]
    x = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    dy = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    rmsnorm_backward(x, w, dy, 1e-6)
    t0 = time.perf_counter()
    reps = 0
    while True:
        rmsnorm_backward(x, w, dy, 1e-6)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(rmsnorm_bwd_bytes(rows, hidden) / dt / 1e9, 3), "unit": "GB/s", "cores": cores,
            "kind": "port", "sample": f"{rows} x {hidden} bf16 rows, {reps} passes, oracle/rmsnorm.py "
                                      f"rmsnorm_backward (torch float64 autograd on the CPU, {cores} threads)"}


# ---------------------------------------------------------------------------------------------
# SANA linear attention
# ---------------------------------------------------------------------------------------------
def sana_bytes(cfg):
    c = cfg["H"] * cfg["D"]
    return 2 * cfg["B"] * cfg["N"] * 3 * c + 2 * cfg["B"] * cfg["N"] * c


def bench_sana(args, dist, peaks, peak_kind, cfg):
    from kernelforge_b200.SANA_LinearAttention import qkv_attn_matmul

    dev = torch.device("cuda", torch.cuda.current_device())
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    gen = torch.Generator(device=dev).manual_seed(77 + dist.rank)
    one = 2 * B * N * 3 * H * D
    copies = max(1, math.ceil(2 * L2_BYTES / one))  # rotate inputs so each step's data is not L2-hot
    qkvs = [torch.randn(B, N, 3, H * D, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(copies)]
    fn = qkv_attn_matmul(B, H, D, N, dtype="bfloat16", output_dtype="bfloat16")
    # One call is one or two launches of tens of microseconds: the device-resident number replays
    # calls from CUDA graphs so that it measures the kernels, not Python or graph launches. A
    # replay runs `cpg` consecutive calls (one call = one step) on rotating inputs; the timed
    # region is exactly args.steps calls. e2e below keeps the plain per-call API.
    cpg = max(c for c in range(1, 11) if args.steps % c == 0)
    outs = [fn(q) for q in qkvs]
    torch.cuda.synchronize()
    graphs = []
    for gi in range(copies):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for c in range(cpg):
                outs.append(fn(qkvs[(gi * cpg + c) % copies]))
        graphs.append(g)
    timer = LaunchTimer()

    def step(i):
        timer.around(graphs[i % copies].replay)

    ms, dom_ms = time_region(step, args.steps // cpg, -(-args.warmup // cpg), dist, timer)
    ms, dom_ms = ms / cpg, dom_ms / cpg
    nbytes = sana_bytes(cfg)
    value = dist.world * nbytes / (ms / 1e3) / 1e9
    flops = 4 * B * H * N * D * (D + 1)
    launches = sana_launches_per_call(B, H, N)
    result = {
        "value": round(value, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "gpu_launches": launches * args.steps,
        "config": {"B": B, "H": H, "N": N, "D": D, "dtype_in": "bf16", "dtype_out": "bf16",
                   "input_copies": copies, "l2": f"{copies} rotating qkv copies ({copies * one / 1e6:.0f} MB)",
                   "launch": f"CUDA graphs of {cpg} consecutive qkv_attn_matmul calls (one call = one step)"},
        "roofline": roofline(nbytes, dom_ms, peaks["hbm_gbs"], "GB/s", "hbm",
                             SANA_NCU_TRAFFIC_BYTES.get(cfg["name"])),
        "roofline_note": f"{'the one-launch kernel' if launches == 1 else 'producer + epilogue launches'} of one "
                         f"call, {dom_ms * 1e3:.1f} us avg over graph replays; "
                         f"{flops / (dom_ms / 1e3) / 1e12:.1f} TFLOP/s of algorithmic FMA work; "
                         f"peak = {peak_kind} HBM copy GB/s",
    }
    if not args.no_e2e:
        host_in = torch.empty(qkvs[0].shape, dtype=torch.bfloat16, pin_memory=True)
        host_out = torch.empty(B, N, H * D, dtype=torch.bfloat16, pin_memory=True)
        dev_in = torch.empty_like(qkvs[0])

        def e2e_step(_):
            dev_in.copy_(host_in, non_blocking=True)
            host_out.copy_(fn(dev_in), non_blocking=True)

        steps = max(3, min(args.steps, 4 * args.e2e_steps))
        ems, _ = time_region(e2e_step, steps, args.warmup, dist)
        result["e2e"] = {"value": round(dist.world * nbytes / (ems / 1e3) / 1e9, 2), "unit": "GB/s",
                         "h2d_bytes_per_step": host_in.numel() * 2, "d2h_bytes_per_step": host_out.numel() * 2,
                         "steps": steps, "ms_per_step": round(ems, 4),
                         "api": "kernelforge_b200.SANA_LinearAttention.qkv_attn_matmul(...)(qkv)"}
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = sana_cpu_baseline(cfg, seconds=args.cpu_seconds / 2)
    del qkvs, outs, graphs
    torch.cuda.empty_cache()
    return result


def sana_cpu_baseline(cfg, seconds=5.0):
    """oracle.sana (the reference's attn_matmul, bf16 matmuls) over a bounded token sample."""
    from oracle.sana import qkv_attention_reference

    cores = cpu_threads()
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    n = min(N, 4096)
    g = torch.Generator().manual_seed(0)
    qkv = torch.randn(1, n, 3, H * D, generator=g).to(torch.bfloat16)
    qkv_attention_reference(qkv, H, D)
    t0 = time.perf_counter()
    reps = 0
    while True:
        qkv_attention_reference(qkv, H, D)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    nbytes = sana_bytes(dict(cfg, B=1, N=n))
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"B=1, N={n} of (B={B},H={H},N={N},D={D}), {reps} passes, oracle/sana.py "
                      f"(reference attn_matmul on torch CPU, {cores} threads)"}


# ---------------------------------------------------------------------------------------------
# FlashAttention JVP (B=4, H=16, N=4096, D in {64, 128}, bf16, non-causal)
# ---------------------------------------------------------------------------------------------
FA_CONFIGS = (
    {"name": "fajvp_d64", "B": 4, "H": 16, "N": 4096, "D": 64},
    {"name": "fajvp_d128", "B": 4, "H": 16, "N": 4096, "D": 128},
)
FA_SMALL = (
    {"name": "fajvp_d64", "B": 1, "H": 8, "N": 4096, "D": 64},
    {"name": "fajvp_d128", "B": 1, "H": 8, "N": 4096, "D": 128},
)


def fa_flops(cfg, gemms):
    return 2 * gemms * cfg["B"] * cfg["H"] * cfg["N"] * cfg["N"] * cfg["D"]


def bench_fa(args, dist, peaks, peak_kind, cfg, fused):
    import kernelforge_b200.flash_attention_jvp as fa

    dev = torch.device("cuda", torch.cuda.current_device())
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    gen = torch.Generator(device=dev).manual_seed(2026 + dist.rank)
    q, k, v, tq, tk, tv = (torch.randn(B, N, H, D, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(6))
    out, lse = fa.flash_attention(q, k, v, return_lse=True)
    if fused:
        call = lambda: fa.flash_attention_fwd_jvp(q, k, v, tq, tk, tv)  # noqa: E731
        gemms, what = 6, "one-pass O, LSE and tangent (flash_attention_fwd_jvp)"
    else:
        call = lambda: fa.flash_attention_jvp(q, k, v, tq, tk, tv, out, lse)  # noqa: E731
        gemms, what = 5, "standalone tangent from cached O/LSE (flash_attention_jvp)"
    timer = LaunchTimer()
    keep = []

    def step(_):
        keep.append(timer.around(call))
        if len(keep) > 2:
            keep.pop(0)

    ms, dom_ms = time_region(step, args.steps, args.warmup, dist, timer)
    flops = fa_flops(cfg, gemms)
    peak = peaks["bf16_tflops"]
    result = {
        "value": round(dist.world * flops / (ms / 1e3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "gpu_launches": args.steps,
        "config": {"B": B, "H": H, "N": N, "D": D, "causal": False, "dtype": "bf16", "call": what,
                   "flops_per_step": flops, "l2": "inputs larger than L2 (6-8 tensors of B*N*H*D bf16)"},
        "roofline": roofline(flops, dom_ms, peak, "TFLOP/s", "tensor"),
        "roofline_note": f"{gemms} GEMMs x 2*B*H*N^2*D flop per launch, {dom_ms * 1e3:.1f} us avg; "
                         f"peak = {peak_kind} cuBLAS bf16 TFLOP/s (burst)",
    }
    if not args.no_e2e:
        host = [torch.empty_like(t, device="cpu").pin_memory() for t in (q, k, v, tq, tk, tv)]
        for h, t in zip(host, (q, k, v, tq, tk, tv)):
            h.copy_(t)
        host_out = torch.empty_like(q, device="cpu").pin_memory()
        dev_in = [torch.empty_like(t) for t in (q, k, v, tq, tk, tv)]
        h2d = sum(t.numel() * 2 for t in host)
        if not fused:
            host_o = out.cpu().pin_memory()
            host_lse = lse.cpu().pin_memory()
            dev_o, dev_lse = torch.empty_like(out), torch.empty_like(lse)
            h2d += host_o.numel() * 2 + host_lse.numel() * 4

        def e2e_step(_):
            for d_, h_ in zip(dev_in, host):
                d_.copy_(h_, non_blocking=True)
            if fused:
                _, _, tangent = fa.flash_attention_fwd_jvp(*dev_in)
            else:
                dev_o.copy_(host_o, non_blocking=True)
                dev_lse.copy_(host_lse, non_blocking=True)
                tangent = fa.flash_attention_jvp(*dev_in, dev_o, dev_lse)
            host_out.copy_(tangent, non_blocking=True)

        steps = max(3, min(args.steps, args.e2e_steps))
        ems, _ = time_region(e2e_step, steps, args.warmup, dist)
        result["e2e"] = {"value": round(dist.world * flops / (ems / 1e3) / 1e12, 2), "unit": "TFLOP/s",
                         "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": host_out.numel() * 2,
                         "steps": steps, "ms_per_step": round(ems, 3),
                         "api": "kernelforge_b200.flash_attention_jvp." +
                                ("flash_attention_fwd_jvp" if fused else "flash_attention_jvp")}
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = fa_cpu_baseline(cfg, fused, seconds=args.cpu_seconds / 2)
    del q, k, v, tq, tk, tv, out, lse, keep
    torch.cuda.empty_cache()
    return result


def fa_cpu_baseline(cfg, fused, seconds=5.0):
    """oracle.fa_jvp on the host cores, one (batch, head) slice of the config at a time."""
    from oracle.fa_jvp import attention_jvp, attention_jvp_from_forward, attention_lse, attention

    cores = cpu_threads()
    N, D = cfg["N"], cfg["D"]
    g = torch.Generator().manual_seed(0)
    q, k, v, tq, tk, tv = (torch.randn(1, N, 1, D, generator=g).to(torch.bfloat16) for _ in range(6))
    if not fused:
        out = attention(q, k, v)
        lse = attention_lse(q, k)
    t0 = time.perf_counter()
    reps = 0
    while True:
        if fused:
            attention_jvp(q, k, v, tq, tk, tv)
        else:
            attention_jvp_from_forward(q, k, v, tq, tk, tv, out, lse)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    flops = fa_flops(dict(cfg, B=1, H=1), 6 if fused else 5)
    return {"value": round(flops / dt / 1e12, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{reps} (batch, head) slices of N={N}, D={D} (of B={cfg['B']}, H={cfg['H']}), "
                      f"oracle/fa_jvp.py {'attention_jvp (torch.func)' if fused else 'attention_jvp_from_forward'} "
                      f"on torch CPU fp32, {cores} threads"}


# ---------------------------------------------------------------------------------------------
# FlashAttention backward (FlashAttentionFunction.backward -> _flash_attn_backward), same configs
# ---------------------------------------------------------------------------------------------
FA_BWD_CONFIGS = tuple(dict(c, name=c["name"].replace("fajvp", "fabwd")) for c in FA_CONFIGS)
FA_BWD_SMALL = tuple(dict(c, name=c["name"].replace("fajvp", "fabwd")) for c in FA_SMALL)


def flash_attn_backward_tflops(q, k, v, out, lse, dout, scale, flops, steps=10):
    """The flash_attn binary's backward on the same tensors (what the reference's
    FlashAttentionFunction.backward calls); context only, None when it cannot run."""
    try:
        from flash_attn.flash_attn_interface import _flash_attn_backward as fa_bwd
    except Exception:
        return None
    dq, dk, dv = (torch.empty_like(x) for x in (q, k, v))

    def call():
        fa_bwd(dout, q, k, v, out, lse, dq, dk, dv, 0.0, scale, False, -1, -1, 0.0, None, False)

    try:
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            call()
        b.record()
        b.synchronize()
    except Exception:
        return None
    return round(flops / (a.elapsed_time(b) / steps / 1e3) / 1e12, 1)


def bench_fa_bwd(args, dist, peaks, peak_kind, cfg):
    from kernelforge_b200.flash_attention_jvp import custom as fa

    dev = torch.device("cuda", torch.cuda.current_device())
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    scale = D ** -0.5
    gen = torch.Generator(device=dev).manual_seed(2026 + dist.rank)
    q, k, v, dout = (torch.randn(B, N, H, D, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(4))
    out, lse = fa.flash_attention(q, k, v, return_lse=True)
    dq, dk, dv = (torch.empty_like(x) for x in (q, k, v))
    call = lambda: fa._flash_attn_backward(dout, q, k, v, out, lse, dq, dk, dv, 0.0, scale, False)  # noqa: E731
    timer = LaunchTimer()
    ms, dom_ms = time_region(lambda _: timer.around(call), args.steps, args.warmup, dist, timer)
    flops = fa_flops(cfg, 5)
    peak = peaks["bf16_tflops"]
    result = {
        "value": round(dist.world * flops / (ms / 1e3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "gpu_launches": 3 * args.steps,
        "config": {"B": B, "H": H, "N": N, "D": D, "causal": False, "dtype": "bf16",
                   "call": "_flash_attn_backward (dq, dk, dv from dout and the saved O, LSE)",
                   "flops_per_step": flops, "l2": "inputs larger than L2 (8 tensors of B*N*H*D bf16)"},
        "roofline": roofline(flops, dom_ms, peak, "TFLOP/s", "tensor"),
        "roofline_note": f"5 GEMMs x 2*B*H*N^2*D algorithmic flop per call (the kernels recompute S and dP in "
                         f"both the dQ and the dK/dV kernel: 7 GEMMs executed); one call = 3 launches "
                         f"(row statistics, dQ, dK/dV), {dom_ms * 1e3:.1f} us avg per call; "
                         f"peak = {peak_kind} cuBLAS bf16 TFLOP/s (burst)",
    }
    if dist.rank == 0 and args.flash_attn_comparator:
        result["flash_attn_backward_tflops"] = flash_attn_backward_tflops(q, k, v, out, lse, dout, scale, flops)
    if not args.no_e2e:
        host = [t.cpu().pin_memory() for t in (dout, q, k, v, out)]
        host_lse = lse.cpu().pin_memory()
        dev_in = [torch.empty_like(t) for t in (dout, q, k, v, out)]
        dev_lse = torch.empty_like(lse)
        host_grads = [torch.empty_like(t, device="cpu").pin_memory() for t in (dq, dk, dv)]
        h2d = sum(t.numel() * 2 for t in host) + host_lse.numel() * 4

        def e2e_step(_):
            for d_, h_ in zip(dev_in, host):
                d_.copy_(h_, non_blocking=True)
            dev_lse.copy_(host_lse, non_blocking=True)
            fa._flash_attn_backward(*dev_in, dev_lse, dq, dk, dv, 0.0, scale, False)
            for h_, g_ in zip(host_grads, (dq, dk, dv)):
                h_.copy_(g_, non_blocking=True)

        steps = max(3, min(args.steps, args.e2e_steps))
        ems, _ = time_region(e2e_step, steps, args.warmup, dist)
        result["e2e"] = {"value": round(dist.world * flops / (ems / 1e3) / 1e12, 2), "unit": "TFLOP/s",
                         "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": sum(t.numel() * 2 for t in host_grads),
                         "steps": steps, "ms_per_step": round(ems, 3),
                         "api": "kernelforge_b200.flash_attention_jvp.custom._flash_attn_backward"}
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = fa_bwd_cpu_baseline(cfg, seconds=args.cpu_seconds / 2)
    del q, k, v, dout, out, lse, dq, dk, dv
    torch.cuda.empty_cache()
    return result


def fa_bwd_cpu_baseline(cfg, seconds=5.0):
    """Float32 autograd through oracle.fa_jvp.attention on the host cores, one (batch, head) slice
    of the config at a time."""
    from oracle.fa_jvp import attention

    cores = cpu_threads()
    N, D = cfg["N"], cfg["D"]
    g = torch.Generator().manual_seed(0)
    q, k, v, dout = (torch.randn(1, N, 1, D, generator=g) for _ in range(4))
    t0 = time.perf_counter()
    reps = 0
    while True:
        primals = tuple(x.clone().requires_grad_() for x in (q, k, v))
        torch.autograd.grad(attention(*primals), primals, dout)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    flops = fa_flops(dict(cfg, B=1, H=1), 5)
    return {"value": round(flops / dt / 1e12, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{reps} (batch, head) slices of N={N}, D={D} (of B={cfg['B']}, H={cfg['H']}), "
                      f"torch.autograd through oracle/fa_jvp.py attention on torch CPU fp32, {cores} threads"}


# ---------------------------------------------------------------------------------------------
# reference arm: the reference algorithm on the host cores (oracle restatement)
# ---------------------------------------------------------------------------------------------
def run_reference(args):
    from oracle.rmsnorm import rmsnorm_forward

    cores = cpu_threads()
    g = torch.Generator().manual_seed(0)
    rows = rmsnorm_cpu_sample_rows()
    data = [(torch.randn(min(rows, r), h, generator=g).to(torch.bfloat16),
             (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16)) for r, h in sweep_points()]
    nbytes = sum(rmsnorm_bytes(x.shape[0], x.shape[1]) for x, _ in data)

    def step():
        for x, w in data:
            rmsnorm_forward(x, w, 1e-6)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = round(nbytes / dt / 1e9, 3)
    sample = (f"first {rows} rows of each of the 12 RMSNorm sweep tensors per step "
              f"({nbytes / 1e6:.0f} MB), oracle/rmsnorm.py on torch CPU")
    line = {
        "impl": "reference", "metric": BASELINE_METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "rmsnorm_bf16_sweep (bounded CPU sample)", "rows": list(SWEEP_ROWS),
                   "hidden": list(SWEEP_HIDDEN), "sample_rows": rows},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("all", "rmsnorm", "rmsnormbwd", "sana", "fajvp", "fabwd"), default="all")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--flash-attn-comparator", action="store_true",
                    help="also time the flash_attn binary's backward on the fabwd tensors (context only; "
                         "off by default so that the default run loads no attention library)")
    ap.add_argument("--case", choices=("full", "ncu-small"), default="full",
                    help="ncu-small: one small configuration per workload, for ncu --set full captures")
    args = ap.parse_args()
    global CASE
    CASE = args.case
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    dist = Dist()
    if args.impl == "reference":
        if dist.rank == 0:
            run_reference(args)
        return
    dist.init()
    peaks, peak_kind = load_peaks()
    sampler = ClockSampler(dist.local_rank)
    sampler.start()
    workloads = {}
    head = None
    if args.workload in ("all", "rmsnorm"):
        head = bench_rmsnorm(args, dist, peaks, peak_kind)
    if args.workload in ("all", "rmsnormbwd"):
        workloads["rmsnormbwd_bf16_32768x8192"] = bench_rmsnorm_bwd(args, dist, peaks, peak_kind)
    if args.workload in ("all", "sana"):
        for cfg in (SANA_CONFIGS[:1] if CASE == "ncu-small" else SANA_CONFIGS):
            workloads[cfg["name"]] = bench_sana(args, dist, peaks, peak_kind, cfg)
    if args.workload in ("all", "fajvp"):
        for cfg in (FA_SMALL if CASE == "ncu-small" else FA_CONFIGS):
            workloads[cfg["name"] + "_standalone"] = bench_fa(args, dist, peaks, peak_kind, cfg, fused=False)
            workloads[cfg["name"] + "_fused"] = bench_fa(args, dist, peaks, peak_kind, cfg, fused=True)
    if args.workload in ("all", "fabwd"):
        for cfg in (FA_BWD_SMALL if CASE == "ncu-small" else FA_BWD_CONFIGS):
            workloads[cfg["name"]] = bench_fa_bwd(args, dist, peaks, peak_kind, cfg)
    clocks = sampler.stop()
    if head is None:  # a single secondary workload was requested: promote it
        name, head = next(iter(workloads.items()))
        workload_name = name
    else:
        workload_name = "rmsnorm_bf16_sweep"
    if dist.rank == 0:
        line = {
            "metric": BASELINE_METRIC, "value": head["value"], "unit": head["unit"],
            "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) tensors generated on device)",
            "config": {"workload": workload_name if CASE == "full" else workload_name + " (ncu-small case)",
                       "rows": sorted({r for r, _ in sweep_points()}),
                       "hidden": sorted({h for _, h in sweep_points()}),
                       "eps": 1e-6, "l2": "inputs larger than L2: one step streams every sweep tensor",
                       "parallelism": f"weak scaling, {dist.world} rank(s) x full sweep, no collective"},
            "roofline": head["roofline"], "gpu_launches": head["gpu_launches"],
            "peaks": {"kind": peak_kind, "hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": peaks["bf16_tflops"]},
        }
        for key in ("e2e", "cpu_baseline", "roofline_note"):
            if key in head:
                line[key] = head[key]
        if clocks:
            line["clocks"] = clocks
        line["workloads"] = workloads
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
